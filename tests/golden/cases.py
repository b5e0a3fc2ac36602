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
