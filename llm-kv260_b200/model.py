"""Random-init Llama-shaped Q4_0 models (no checkpoints here): seeded GGUF
Q4_0 bytes for every linear, in the tensor layout a GGUF file holds and the
reference's loader reads (board/tp/tp_llama.cpp:226-283).

Weights: uniform nibbles and float16 scales 0.0043 * U(0.75, 1.25), so the
weights spread about like N(0, 0.02); RMSNorm weights 1 + 0.05 * N(0, 1);
no rope frequency factors; the embedding table is also the (tied) lm_head.
"""

from __future__ import annotations

import numpy as np

# BASELINE configurations (hparams of board/tp/tp_llama.cpp:123-126)
LLAMA_1B = dict(n_layer=16, n_embd=2048, n_ff=8192, n_head=32, n_head_kv=8, head_dim=64, n_vocab=128256,
                rope_base=500000.0, rms_eps=1e-5)
LLAMA_3B = dict(n_layer=28, n_embd=3072, n_ff=8192, n_head=24, n_head_kv=8, head_dim=128, n_vocab=128256,
                rope_base=500000.0, rms_eps=1e-5)


def q4_0_rows(rng: np.random.Generator, rows: int, k: int) -> np.ndarray:
    """[rows, k/32*18] uint8: seeded Q4_0 blocks (fp16 scale, then 16 nibble bytes)."""
    nb = k // 32
    raw = rng.integers(0, 256, size=(rows * nb, 18), dtype=np.uint8)
    d = (0.0043 * (0.75 + 0.5 * rng.random(rows * nb))).astype(np.float16)
    raw[:, 0:2] = d.view(np.uint8).reshape(-1, 2)
    return raw.reshape(rows, nb * 18)


def synth_model(hp: dict, seed: int = 0) -> dict:
    """A full (unsharded) model: hparams plus "layers" (attn_q, attn_k, attn_v,
    attn_output, ffn_gate, ffn_up, ffn_down as Q4_0 rows; attn_norm, ffn_norm
    float32), "token_embd" and "output_norm"."""
    rng = np.random.default_rng(seed)
    e, f, kv = hp["n_embd"], hp["n_ff"], hp["n_head_kv"] * hp["head_dim"]

    def norm() -> np.ndarray:
        return (1.0 + 0.05 * rng.standard_normal(e)).astype(np.float32)

    layers = []
    for _ in range(hp["n_layer"]):
        layers.append(dict(attn_q=q4_0_rows(rng, e, e), attn_k=q4_0_rows(rng, kv, e), attn_v=q4_0_rows(rng, kv, e),
                           attn_output=q4_0_rows(rng, e, e), ffn_gate=q4_0_rows(rng, f, e),
                           ffn_up=q4_0_rows(rng, f, e), ffn_down=q4_0_rows(rng, e, f), attn_norm=norm(),
                           ffn_norm=norm()))
    model = dict(hp)
    model.update(layers=layers, token_embd=q4_0_rows(rng, hp["n_vocab"], e), output_norm=norm())
    return model


def random_prompt(n: int, n_vocab: int, seed: int = 0) -> np.ndarray:
    """n uniform-random token ids (BASELINE's prompts)."""
    return np.random.default_rng(seed).integers(0, n_vocab, size=n, dtype=np.int32)
