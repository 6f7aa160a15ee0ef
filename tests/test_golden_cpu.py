"""Golden fixtures from the reference's own Python modules (CPU only).

  plain_block_t8.npz    fhe/realweights/manual.py block_reference  -> pins
                        oracle/plain_block.py (the decrypted-output checker)
  plain_head.npz        fhe/multiblock/manual.py classifier_head_reference
                        (readout rows N, A) -> pins oracle/plain_block.py
                        head() and its N - A margin
  simd_layout_b32.*     fhe/gpu_real_scheme_b/simd_layout.py at 32 tokens per
                        ciphertext, one copy -> pins the engine's host-side
                        block schedule (causal lane shifts, BSGS diagonals)
Fixture generator: tests/golden/make_golden.py.
"""

import json
import os

import numpy as np

import private_genomic_dnagpt_b200 as eng
from oracle import plain_block
from tests.golden.inputs import layout_inputs

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_plain_block_oracle_matches_reference_manual_py():
    g = np.load(os.path.join(GOLD, "plain_block_t8.npz"))
    w = plain_block.synthetic_weights(int(g["seed_weights"]))
    x = plain_block.synthetic_input(int(g["seed_input"]), 8)
    got = plain_block.block(x, w, return_all=True)
    for k in ("block_output", "ln1_output", "attention_scores", "residual1"):
        ref = g[k]
        assert np.abs(got[k] - ref).max() <= 1e-12 * max(1.0, np.abs(ref).max()), k


def test_plain_head_oracle_matches_reference_manual_py():
    g = np.load(os.path.join(GOLD, "plain_head.npz"))
    hw = plain_block.synthetic_head_weights(int(g["seed_weights"]))
    hidden = plain_block.synthetic_input(int(g["seed_hidden"]), 4)
    assert np.abs(g["readout_rows"][0] - g["readout_rows"][1] - hw["readout"]).max() < 1e-15
    for t in range(4):
        m = plain_block.head(hidden[t], hw)
        assert abs(m - g["margin"][t]) <= 1e-12 * max(1.0, abs(g["margin"][t])), t
    # a two-block model ends in the same head on its last token
    w = [plain_block.synthetic_weights(3), plain_block.synthetic_weights(4)]
    x = plain_block.synthetic_input(4, 5)
    h, m = plain_block.model(x, w, hw)
    assert np.allclose(h, plain_block.block(plain_block.block(x, w[0]), w[1]), rtol=0, atol=0)
    assert m == plain_block.head(h[-1], hw)


def test_causal_lane_shifts_match_simd_layout():
    gold = json.load(open(os.path.join(GOLD, "simd_layout_b32.json")))
    T, B = gold["tokens"], gold["batch_width"]
    total = 0
    for key, shifts in gold["active_weight_shifts"].items():
        qg, kg = map(int, key.split(","))
        got = eng.schedule_active_shifts(T, B, qg, kg)
        assert got == shifts, key
        total += len(got)
    assert total == gold["protocol_counts"]["weight_tile_encryptions"]
    for c, f, t, slot in gold["slots"]:
        assert f * B + t == slot  # slot(feature, lane) = feature * B + lane (one copy)


def _rot(v, k):
    return np.roll(v, -k)


def test_bsgs_diagonals_reproduce_simd_layout_transform():
    g = np.load(os.path.join(GOLD, "simd_layout_b32.npz"))
    tok, W, *_ = layout_inputs()
    B, PW, n1, dim = 32, 64, 8, 48
    n2 = PW // n1
    x = np.zeros((PW, B))
    x[:dim, : tok.shape[0]] = tok.T
    x = x.reshape(-1)
    y = np.zeros_like(x)
    for gg in range(n2):
        inner = np.zeros_like(x)
        for j in range(n1):
            inner += eng.schedule_diagonal(W, dim, dim, PW, B, n1, gg, j) * _rot(x, B * j)
        y += _rot(inner, B * n1 * gg)
    assert np.abs(y - g["bsgs_out"]).max() < 1e-9


def test_lane_shift_formula_matches_simd_layout():
    """Two rotations and two complementary lane masks (the engine's lane_shift)."""
    g = np.load(os.path.join(GOLD, "simd_layout_b32.npz"))
    v = g["lane_shift_in"]
    B = 32
    lane = np.arange(v.size) % B
    for d in (0, 1, 5, 31, -3):
        dd = d % B
        got = v.copy() if dd == 0 else np.where(lane < B - dd, _rot(v, dd), _rot(v, dd - B))
        assert np.array_equal(got, g[f"lane_shift_{d}"])
