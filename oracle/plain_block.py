"""Float64 plaintext DNAGPT block and model: the checker for decrypted
block outputs and head margins.

TEST INFRASTRUCTURE ONLY (tests/, smoke(), bench CPU legs).  Restates the
reference's bias-free block oracle, fhe/realweights/manual.py:36-106
(block_reference): pre-LN with gain only (eps 1e-5, manual.py:12-18),
x @ W.T with PyTorch [out, in] weights (:21-22), causal stable softmax
(:25-28, :64-66), tanh-GELU (:31-33), residuals (:70, :78).  Pinned against
that function's own output by tests/golden/plain_block_*.npz.  The classifier
head restates fhe/multiblock/manual.py:41-80 (stable SiLU,
classifier_head_reference) with the N - A readout margin of the 12-block
driver (real_dnagpt_fides_scheme_b_simd_full_t103_12blocks_head_cpudiagcache_
t123_v3.cpp:544-550, 594-597); pinned by tests/golden/plain_head.npz.
"""

from __future__ import annotations

import math

import numpy as np

D, HEADS, HEAD_DIM, MLP = 768, 12, 64, 3072


def layer_norm(x, gain, eps=1e-5):
    mean = x.mean(axis=-1, keepdims=True)
    centered = x - mean
    var = (centered * centered).mean(axis=-1, keepdims=True)
    return centered / np.sqrt(var + eps) * gain


def gelu_tanh(x):
    return 0.5 * x * (1.0 + np.tanh(math.sqrt(2.0 / math.pi) * (x + 0.044715 * x ** 3)))


def block(x, w, heads=HEADS, eps=1e-5, return_all=False):
    """w: dict with ln1 [D], attn_qkv [3D,D], attn_proj [D,D], ln2 [D],
    mlp_fc [4D,D], mlp_proj [D,4D] (float64)."""
    x = np.asarray(x, np.float64)
    T, Dm = x.shape
    hd = Dm // heads
    h1 = layer_norm(x, w["ln1"], eps)
    qkv = h1 @ w["attn_qkv"].T
    q, k, v = (qkv[:, i * Dm:(i + 1) * Dm].reshape(T, heads, hd).transpose(1, 0, 2) for i in range(3))
    scores = q @ k.transpose(0, 2, 1) / math.sqrt(hd)
    mask = np.tril(np.ones((T, T), bool))
    s = np.where(mask[None], scores, -np.inf)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(axis=-1, keepdims=True)
    ctx = (p @ v).transpose(1, 0, 2).reshape(T, Dm)
    r1 = x + ctx @ w["attn_proj"].T
    h2 = layer_norm(r1, w["ln2"], eps)
    fc = h2 @ w["mlp_fc"].T
    out = r1 + gelu_tanh(fc) @ w["mlp_proj"].T
    if return_all:
        return {"ln1_output": h1, "qkv": qkv, "attention_scores": scores, "attention_probabilities": p,
                "residual1": r1, "mlp_fc": fc, "block_output": out}
    return out


def silu(x):
    """Stable SiLU (multiblock/manual.py:41-49)."""
    x = np.asarray(x, np.float64)
    sig = np.empty_like(x)
    pos = x >= 0
    sig[pos] = 1.0 / (1.0 + np.exp(-x[pos]))
    e = np.exp(x[~pos])
    sig[~pos] = e / (1.0 + e)
    return x * sig


def head(hidden_last, hw, eps=1e-5):
    """N - A margin of one hidden state: final LN -> head linear -> SiLU ->
    head LN -> dot with readout (readout = readout_N - readout_A)."""
    f = layer_norm(np.asarray(hidden_last, np.float64), hw["final_ln"], eps)
    lin = f @ hw["head_linear"].T
    hl = layer_norm(silu(lin), hw["head_ln"], eps)
    return float(hl @ hw["readout"])


def model(x, blocks_w, hw=None, heads=HEADS):
    """Chained blocks, then the head on the last token; returns (hidden, margin)."""
    h = np.asarray(x, np.float64)
    for w in blocks_w:
        h = block(h, w, heads)
    return h, (head(h[-1], hw) if hw is not None else None)


def synthetic_head_weights(seed: int, d=D, std=0.02):
    """Head weights: unit LN gains, head linear N(0, std) [out, in], readout
    margin row N(0, std)."""
    rng = np.random.default_rng(seed)
    return {"final_ln": np.ones(d), "head_linear": rng.normal(0.0, std, (d, d)), "head_ln": np.ones(d),
            "readout": rng.normal(0.0, std, d)}


def synthetic_weights(seed: int, d=D, mlp=MLP, std=0.02, gain_jitter=0.0):
    """Random-init weights N(0, std) in [out, in] layout; unit LN gains (the
    reference fixtures export gains only, fhe/multiblock/export_fixture.py:51-59)."""
    rng = np.random.default_rng(seed)
    w = {
        "attn_qkv": rng.normal(0.0, std, (3 * d, d)),
        "attn_proj": rng.normal(0.0, std, (d, d)),
        "mlp_fc": rng.normal(0.0, std, (mlp, d)),
        "mlp_proj": rng.normal(0.0, std, (d, mlp)),
    }
    w["ln1"] = 1.0 + gain_jitter * rng.standard_normal(d)
    w["ln2"] = 1.0 + gain_jitter * rng.standard_normal(d)
    return w


def synthetic_input(seed: int, tokens: int, d=D):
    """Embeddings N(0, 1) clipped to +-4."""
    return np.clip(np.random.default_rng(seed).standard_normal((tokens, d)), -4.0, 4.0)


def rel_inf(ref, got):
    return float(np.max(np.abs(got - ref)) / max(float(np.max(np.abs(ref))), 1e-12))
