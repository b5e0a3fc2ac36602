"""Write a random-init model (llm-kv260_b200/model.py's dict) as a GGUF Q4_0
file with the installed gguf-py (0.19): the llama.* keys and tensor names the
reference's loader reads (board/tp/tp_llama.cpp:226-283). Test helper only."""

from __future__ import annotations

import numpy as np


def write_gguf(model: dict, path: str, rope_freqs: np.ndarray | None = None) -> str:
    import gguf
    w = gguf.GGUFWriter(path, "llama")
    w.add_block_count(int(model["n_layer"]))
    w.add_embedding_length(int(model["n_embd"]))
    w.add_feed_forward_length(int(model["n_ff"]))
    w.add_head_count(int(model["n_head"]))
    w.add_head_count_kv(int(model["n_head_kv"]))
    w.add_vocab_size(int(model["n_vocab"]))
    w.add_rope_freq_base(float(model["rope_base"]))
    w.add_layer_norm_rms_eps(float(model["rms_eps"]))
    q4 = gguf.GGMLQuantizationType.Q4_0
    w.add_tensor("token_embd.weight", np.ascontiguousarray(model["token_embd"]), raw_dtype=q4)
    w.add_tensor("output_norm.weight", np.ascontiguousarray(model["output_norm"], dtype=np.float32))
    if rope_freqs is not None:
        w.add_tensor("rope_freqs.weight", np.ascontiguousarray(rope_freqs, dtype=np.float32))
    for i, L in enumerate(model["layers"]):
        for name in ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"):
            w.add_tensor(f"blk.{i}.{name}.weight", np.ascontiguousarray(L[name]), raw_dtype=q4)
        for name in ("attn_norm", "ffn_norm"):
            w.add_tensor(f"blk.{i}.{name}.weight", np.ascontiguousarray(L[name], dtype=np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return path
