"""Seeded synthetic inputs shared by the fixture generator, the tests and bench.py.

Every input is drawn with numpy's ``default_rng`` (PCG64), so any machine with
numpy regenerates the same float32 arrays. The fixtures in ``golden.json`` hold
SHA-256 digests of what the reference contract (``src/llm_kv260/q4_0.py``)
computed from these inputs, so a test can rebuild the inputs, run the oracle
or the CUDA path, and compare digests without shipping megabytes of floats.
"""

from __future__ import annotations

import hashlib

import numpy as np

# The reference's own golden vector: tests/test_q4_0_contract.py:181-191
# (96 x 2048, standard-normal weights seed 2024, activations seed 2025).
CONTRACT_GOLDEN_SHA256 = "efa9eda8cef689d6392ddf2e1b3e945d19797aff1cbd55398c87ffffec7c29cc"

# hls/int4_core/gen_vectors.py:24-32 cases (k, rows), drawn in this order from
# one default_rng(4) stream (gen_vectors.py:36-41).
GEN_VECTOR_CASES = [(256, 16), (2048, 64), (8192, 16), (256, 32), (8192, 32), (512, 64), (1024, 32)]

# every GEMV shape of one Llama-3.2-1B layer plus lm_head,
# (name, rows N, in_features K, seed). W ~ N(0, 0.02), x ~ N(0, 1).
LLAMA_1B_SHAPES = [
    ("wq", 2048, 2048, 101),
    ("wk", 512, 2048, 102),
    ("wv", 512, 2048, 103),
    ("wo", 2048, 2048, 104),
    ("w1", 8192, 2048, 105),
    ("w3", 8192, 2048, 106),
    ("w2", 2048, 8192, 107),
    ("lm_head", 128256, 2048, 108),
]
# the single 2048 x 2048 GEMV.
CONFIG0 = ("c0", 2048, 2048, 100)

# Matrices split by input columns (row-parallel) across ranks; the rest split
# by output rows (board/tp/tp_llama.cpp:258-279).
K_SPLIT = {"wo", "w2"}
SPLITS = (2, 4, 8)


def sha256(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def std_weights(n: int, k: int, seed: int) -> np.ndarray:
    """The reference tests' `_weights` (tests/test_q4_0_contract.py:29-30)."""
    return np.random.default_rng(seed).standard_normal((n, k)).astype(np.float32)


def shape_weights(n: int, k: int, seed: int) -> np.ndarray:
    """W ~ N(0, 0.02) as float32, drawn in float64 and scaled before the cast."""
    return (np.random.default_rng(seed).standard_normal((n, k)) * 0.02).astype(np.float32)


def shape_x(k: int, seed: int) -> np.ndarray:
    """x ~ N(0, 1) as float32, seed + 1 of the matrix's seed."""
    return np.random.default_rng(seed + 1).standard_normal(k).astype(np.float32)


def gen_vector_inputs():
    """Yield (k, rows, w, x) exactly as gen_vectors.py:36-41 draws them."""
    rng = np.random.default_rng(4)
    for k, rows in GEN_VECTOR_CASES:
        w = rng.standard_normal((rows, k)).astype(np.float32)
        x = rng.standard_normal(k).astype(np.float32)
        yield k, rows, w, x


def k_slice_blocks(blocks: np.ndarray, k: int, r: int, n: int) -> np.ndarray:
    """Columns [r*k/n, (r+1)*k/n) of a Q4_0 matrix: whole 18-byte blocks sliced
    out of every row (tp_llama.cpp:199-207)."""
    kk = k // n
    b0 = r * kk // 32 * 18
    return np.ascontiguousarray(blocks[:, b0:b0 + kk // 32 * 18])


def q8_edge_inputs() -> dict[str, np.ndarray]:
    """Activation blocks whose rounding the contract pins.

    'roundf_tie' is the reference's own test (test_q4_0_contract.py:51-59);
    'floor_half' puts s = 0.5 - 2^-25 and its negative in a block with d = 1,
    where floor(|s| + 0.5f) gives 1 and roundf gives 0."""
    tie = np.zeros(32, dtype=np.float32)
    tie[0], tie[1], tie[2], tie[3] = 127.0, 2.5, -2.5, 0.5
    half = np.zeros(32, dtype=np.float32)
    half[0] = 127.0
    half[1] = np.float32(0.5) - np.float32(2.0 ** -25)
    half[2] = -half[1]
    half[3] = np.float32(1.5)
    half[4] = np.float32(-126.5)
    zero = np.zeros(32, dtype=np.float32)
    negzero = np.full(32, -0.0, dtype=np.float32)
    tiny = np.full(32, 1e-30, dtype=np.float32)
    tiny[::3] = -1e-30
    return {"roundf_tie": tie, "floor_half": half, "zero": zero, "negzero": negzero, "tiny": tiny}


# ------------------------------------------------------------------ decode
# Random-init models run through the reference runtime's own decode code
# (oracle/_ref: tp_llama.cpp's load_model, forward and sample_token compiled
# on the host, float32 KV cache, the runtime's roundf quantiser) by
# gen_ref_decode.py; ref_decode.json holds, per case, the greedy token and
# the SHA-256 of the residual stream after every forward, and every rank's
# logits digest at the last one.

HD64 = dict(n_layer=2, n_embd=512, n_ff=1024, n_head=8, n_head_kv=2, head_dim=64, n_vocab=1024,
            rope_base=500000.0, rms_eps=1e-5)
HD128_G3 = dict(n_layer=2, n_embd=1536, n_ff=1536, n_head=12, n_head_kv=4, head_dim=128, n_vocab=1024,
                rope_base=500000.0, rms_eps=1e-5)
HD64_1L = dict(HD64, n_layer=1)
HD128_G3_1L = dict(HD128_G3, n_layer=1)
TPW = dict(n_layer=2, n_embd=2048, n_ff=8192, n_head=32, n_head_kv=8, head_dim=64, n_vocab=2048,
           rope_base=500000.0, rms_eps=1e-5)
W3B = dict(n_layer=1, n_embd=3072, n_ff=8192, n_head=24, n_head_kv=8, head_dim=128, n_vocab=2048,
           rope_base=500000.0, rms_eps=1e-5)

# name: (hparams, weight seed, ranks, prompt length, positions, gemv2 engine layout, rope_freqs).
# The runtime sizes the engine's output buffer as max(vocab_rows, 2 * ff_rows)
# floats (tp_llama.cpp:1277) and writes n_embd rows into it from the o and down
# GEMVs, so every case keeps 2 * n_ff / ranks >= n_embd.
REF_DECODE_CASES = {
    "hd64_r1": (HD64, 41, 1, 6, 40, False, False),
    "hd64_r2_gemv2": (HD64, 41, 2, 6, 40, True, False),
    "hd128_g3_r1_freqs": (HD128_G3, 42, 1, 5, 24, False, True),
    "hd128_g3_r2_freqs": (HD128_G3, 42, 2, 5, 24, True, True),
    "long_r1": (HD64_1L, 43, 1, 290, 300, False, False),
    # 900 positions of float32 K/V rows at head_dim 128: past what the
    # decoder's cluster attention holds in shared memory, so its streaming
    # attention kernel runs
    "hd128_long_r1": (HD128_G3_1L, 46, 1, 880, 900, False, False),
    "tpw_r4": (TPW, 44, 4, 5, 20, False, False),
    "tpw_r8": (TPW, 44, 8, 5, 20, True, False),
    "w3b_r1": (W3B, 45, 1, 5, 20, False, False),
    "w3b_r4": (W3B, 45, 4, 5, 20, True, False),
}


def rope_freqs(head_dim: int) -> np.ndarray:
    """Llama-3-style frequency factors: 1 for the high frequencies, rising
    smoothly to 8 for the low ones (head_dim/2 float32)."""
    t = np.linspace(0.0, 1.0, head_dim // 2, dtype=np.float64)
    return (1.0 + 7.0 * np.clip((t - 0.3) / 0.5, 0.0, 1.0) ** 2).astype(np.float32)


def ref_decode_model(name: str):
    """(model dict, prompt) of a REF_DECODE_CASES entry."""
    import importlib.util
    import os
    hp, seed, _, n_prompt, _, _, freqs = REF_DECODE_CASES[name]
    here = os.path.dirname(os.path.abspath(__file__))
    spec = importlib.util.spec_from_file_location("b200_case_model", os.path.join(here, "..", "..", "llm-kv260_b200",
                                                                                  "model.py"))
    mdl = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mdl)
    m = mdl.synth_model(hp, seed=seed)
    if freqs:
        m["rope_freqs"] = rope_freqs(hp["head_dim"])
    return m, mdl.random_prompt(n_prompt, hp["n_vocab"], seed=seed + 1000)
