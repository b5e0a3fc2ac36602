"""The library's GGUF reader (include/b200_gguf.h) on files written by the
installed gguf-py: host code only, no GPU. What load_model reads
(board/tp/tp_llama.cpp:149-188, 226-236) must come back unchanged."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import cases
from gguf_model import write_gguf


@pytest.fixture(scope="module")
def model_file(tmp_path_factory, pkg):
    m, _ = cases.ref_decode_model("hd128_g3_r1_freqs")
    path = str(tmp_path_factory.mktemp("gguf") / "m.gguf")
    write_gguf(m, path, rope_freqs=m["rope_freqs"])
    return m, path


def test_hparams_and_tensors_round_trip(pkg, model_file):
    m, path = model_file
    with pkg.GGUFFile(path) as g:
        hp = g.hparams()
        for k in ("n_layer", "n_embd", "n_ff", "n_head", "n_head_kv", "head_dim", "n_vocab"):
            assert hp[k] == m[k], k
        assert np.float32(hp["rope_base"]) == np.float32(m["rope_base"])
        assert np.float32(hp["rms_eps"]) == np.float32(m["rms_eps"])
        for i, L in enumerate(m["layers"]):
            for name in ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"):
                data, typ, ne = g.tensor(f"blk.{i}.{name}.weight")
                assert typ == pkg.gguf.GGML_Q4_0
                rows, rb = L[name].shape
                assert ne[:2] == (rb // 18 * 32, rows)
                assert np.array_equal(data, L[name].reshape(-1))
            for name in ("attn_norm", "ffn_norm"):
                data, typ, ne = g.tensor(f"blk.{i}.{name}.weight")
                assert typ == pkg.gguf.GGML_F32 and ne[0] == m["n_embd"]
                assert np.array_equal(data.view(np.float32), L[name])
        data, typ, _ = g.tensor("token_embd.weight")
        assert np.array_equal(data, m["token_embd"].reshape(-1))
        data, typ, ne = g.tensor("rope_freqs.weight")
        assert typ == pkg.gguf.GGML_F32 and ne[0] == m["head_dim"] // 2
        assert np.array_equal(data.view(np.float32), m["rope_freqs"])
        with pytest.raises(pkg.B200Error):
            g.tensor("blk.99.attn_q.weight")


def test_bad_files_are_refused(pkg, model_file, tmp_path):
    _, path = model_file
    with pytest.raises(pkg.B200Error):
        pkg.GGUFFile(str(tmp_path / "missing.gguf"))
    raw = open(path, "rb").read()
    bad = tmp_path / "bad_magic.gguf"
    bad.write_bytes(b"GGUX" + raw[4:])
    with pytest.raises(pkg.B200Error):
        pkg.GGUFFile(str(bad))
    cut = tmp_path / "truncated.gguf"
    cut.write_bytes(raw[: len(raw) // 2])        # tensors past the end of the file
    with pytest.raises(pkg.B200Error):
        pkg.GGUFFile(str(cut))
    hdr = tmp_path / "header_only.gguf"
    hdr.write_bytes(raw[:40])                     # header cut inside the key/values
    with pytest.raises(pkg.B200Error):
        pkg.GGUFFile(str(hdr))


def test_rope_table_with_frequency_factors_matches_oracle(pkg, oracle):
    from llm_kv260_b200 import decoder
    f = cases.rope_freqs(128)
    for pos in (0, 1, 300, 4351):
        want = oracle.rope_table_freqs(128, pos, 500000.0, f)
        got = decoder.rope_table(128, pos, 500000.0, f)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_config_without_vocab_key_uses_token_embd(pkg, tmp_path):
    """Llama GGUFs converted by llama.cpp carry the vocabulary as tokenizer
    arrays, not always llama.vocab_size; token_embd's rows give it then."""
    import gguf
    m, _ = cases.ref_decode_model("hd64_r1")
    path = str(tmp_path / "novocab.gguf")
    w = gguf.GGUFWriter(path, "llama")
    w.add_block_count(1)
    w.add_embedding_length(m["n_embd"])
    w.add_feed_forward_length(m["n_ff"])
    w.add_head_count(m["n_head"])
    w.add_head_count_kv(m["n_head_kv"])
    w.add_token_list([f"t{i}" for i in range(16)])   # a string array to skip
    w.add_tensor("token_embd.weight", m["token_embd"], raw_dtype=gguf.GGMLQuantizationType.Q4_0)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    with pkg.GGUFFile(path) as g:
        hp = g.hparams()
        assert hp["n_vocab"] == m["n_vocab"] and hp["n_layer"] == 1
        assert np.float32(hp["rope_base"]) == np.float32(10000.0)   # load_model's default
        c = g.config()
        assert ctypes.sizeof(c) > 0
