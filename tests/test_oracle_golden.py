"""Pin the CPU oracle to the reference contract (CPU only).

Every expected value here came from the reference's own ``q4_0.py``
(tests/golden/gen_golden.py) or is the reference's own golden digest
(tests/test_q4_0_contract.py:181 in the reference). The tests mirror the
reference's 13 contract tests (tests/test_q4_0_contract.py) against the
oracle, then add the BASELINE shapes and the rank-ordered K-split sums.
"""

from __future__ import annotations

import numpy as np
import pytest

import cases


def _y(hexstr: str) -> np.ndarray:
    return np.frombuffer(bytes.fromhex(hexstr), dtype=np.float32)


# ----------------------------------------------------------------- float16

def test_f16_to_f32_exhaustive(oracle):
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    want = bits.view(np.float16).astype(np.float32)
    got = np.array([oracle.f16_bits_to_f32(int(h)) for h in bits], dtype=np.float32)
    finite = np.isfinite(want)
    assert np.array_equal(got[finite].view(np.uint32), want[finite].view(np.uint32))
    assert np.all(np.isnan(got[np.isnan(want)]))
    assert np.array_equal(got[np.isinf(want)], want[np.isinf(want)])


def test_f32_to_f16_rounds_to_nearest_even(oracle):
    rng = np.random.default_rng(0)
    vals = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * np.float32(3.0),
        (rng.standard_normal(5000) * 1e-5).astype(np.float32),        # float16 subnormals
        (rng.standard_normal(5000) * 3e4).astype(np.float32),         # near overflow
        # exact ties between float16 neighbours, both parities
        (np.arange(1024, 2048, dtype=np.float32) + np.float32(0.5)),
        np.array([65504.0, 65519.99, 65520.0, 1e9, 2.0 ** -25, 2.0 ** -25 * 1.0001, 2.0 ** -26,
                  5.9604645e-08, -0.0, 0.0], dtype=np.float32),
    ])
    want = vals.astype(np.float16).view(np.uint16)
    got = np.array([oracle.f32_to_f16_bits(float(v)) for v in vals], dtype=np.uint16)
    assert np.array_equal(got, want)


# --------------------------------------------------- codec (reference :35-97)

def test_q4_0_bytes_match_reference(oracle, golden):
    assert cases.sha256(oracle.quantize_q4_0(cases.std_weights(16, 256, 0))) == \
        golden["q4_codec"]["sha256_blocks_16x256_seed0"]


def test_q8_0_bytes_match_reference(oracle, golden):
    q, d = oracle.quantize_q8_0(cases.std_weights(1, 8192, 1)[0])
    assert cases.sha256(q) == golden["q8_random"]["sha256_q"]
    assert cases.sha256(d) == golden["q8_random"]["sha256_d"]


@pytest.mark.parametrize("name", sorted(cases.q8_edge_inputs()))
def test_q8_0_rounding_edges(oracle, golden, name):
    """roundf-style ties (reference :51-59) and the floor(|s|+0.5f) edge at 0.5-2^-25."""
    x = cases.q8_edge_inputs()[name]
    q, d = oracle.quantize_q8_0(x)
    assert q.tolist() == golden["q8_edges"][name]["q"]
    assert d.view(np.uint16).tolist() == golden["q8_edges"][name]["d_bits"]


def test_q8_0_contract_rounding_differs_from_roundf_at_one_value(oracle):
    x = cases.q8_edge_inputs()["floor_half"]
    qc, _ = oracle.quantize_q8_0(x, oracle.ROUND_CONTRACT)
    qr, _ = oracle.quantize_q8_0(x, oracle.ROUND_ROUNDF)
    assert (qc[1], qc[2]) == (1, -1) and (qr[1], qr[2]) == (0, 0)
    assert np.array_equal(np.delete(qc, [1, 2]), np.delete(qr, [1, 2]))


def test_dequantize_and_unpack_match_reference(oracle, golden):
    blocks = oracle.quantize_q4_0(cases.std_weights(8, 512, 2))
    assert cases.sha256(oracle.dequantize_q4_0(blocks, 512)) == golden["q4_codec"]["sha256_dequant_8x512_seed2"]
    ints, d = oracle.unpack_q4_0(blocks, 512)
    assert cases.sha256(ints) == golden["q4_codec"]["sha256_unpack_ints_8x512_seed2"]
    assert cases.sha256(d) == golden["q4_codec"]["sha256_unpack_d_8x512_seed2"]


def test_nibble_layout_is_low_then_high_half_block(oracle):
    row = np.zeros((1, 18), dtype=np.uint8)
    row[0, :2] = np.array([1.0], dtype=np.float16).view(np.uint8)
    row[0, 2] = 0x0F | (0x00 << 4)
    row[0, 3] = 0x08 | (0x09 << 4)
    ints, d = oracle.unpack_q4_0(row, 32)
    assert d[0, 0] == np.float16(1.0)
    assert ints[0, 0] == 7 and ints[0, 16] == -8
    assert ints[0, 1] == 0 and ints[0, 17] == 1


def test_codec_rejects_wrong_inputs(oracle):
    with pytest.raises(TypeError):
        oracle.quantize_q4_0(np.zeros((2, 32), dtype=np.float64))
    with pytest.raises(TypeError):
        oracle.quantize_q8_0(np.zeros(32, dtype=np.float64))
    with pytest.raises(ValueError):
        oracle.quantize_q8_0(np.zeros(33, dtype=np.float32))
    with pytest.raises(ValueError):
        oracle.unpack_q4_0(np.zeros((1, 17), dtype=np.uint8), 32)


# ------------------------------------------------------ gemv (reference :102-191)

def test_golden_vector(oracle):
    """The reference's own frozen digest, through the oracle."""
    w = cases.std_weights(96, 2048, 2024)
    x = cases.std_weights(1, 2048, 2025)[0]
    y = oracle.gemv_q4_0_f32(oracle.quantize_q4_0(w), 2048, x)
    assert cases.sha256(y) == cases.CONTRACT_GOLDEN_SHA256


def test_gen_vector_cases(oracle, golden):
    """hls/int4_core/gen_vectors.py's cases, byte for byte (blocks, x buffer, y)."""
    for (k, rows, w, x), rec in zip(cases.gen_vector_inputs(), golden["gen_vectors"]):
        assert (k, rows) == (rec["k"], rec["rows"])
        blocks = oracle.quantize_q4_0(w)
        xq, xd = oracle.quantize_q8_0(x)
        xp = oracle.pack_x_for_engine(xq, xd)
        assert cases.sha256(blocks) == rec["sha256_blocks"]
        assert cases.sha256(xp) == rec["sha256_xpacked"]
        assert np.array_equal(oracle.gemv_q4_0(blocks, k, xq, xd).view(np.uint32), _y(rec["y"]).view(np.uint32))
        assert np.array_equal(oracle.gemv_q4_0_packed(blocks, k, xp).view(np.uint32), _y(rec["y"]).view(np.uint32))


def test_gemv_is_exact_when_only_one_lane_is_populated(oracle, golden):
    blocks = oracle.quantize_q4_0(cases.std_weights(4, 256, 7))
    xq, xd = oracle.quantize_q8_0(cases.std_weights(1, 256, 8)[0])
    assert np.array_equal(oracle.gemv_q4_0(blocks, 256, xq, xd).view(np.uint32), _y(golden["one_lane"]["y"]).view(np.uint32))


def test_lane_order_is_observable(oracle, golden):
    k = 2048
    blocks = oracle.quantize_q4_0(cases.std_weights(256, k, 9))
    xq, xd = oracle.quantize_q8_0(cases.std_weights(1, k, 10)[0])
    ours = oracle.gemv_q4_0(blocks, k, xq, xd)
    assert cases.sha256(ours) == golden["lane_order"]["sha256_y"]
    ints, dw = oracle.unpack_q4_0(blocks, k)
    nb = k // 32
    sumi = (ints.reshape(256, nb, 32).astype(np.int32) * xq.reshape(nb, 32).astype(np.int32)).sum(-1, dtype=np.int32)
    t = (sumi.astype(np.float32) * dw.astype(np.float32)) * xd.astype(np.float32)
    seq = np.zeros(256, dtype=np.float32)
    for b in range(nb):
        seq = seq + t[:, b]
    assert np.count_nonzero(ours.view(np.uint32) != seq.view(np.uint32)) > 0


def test_gemv_agrees_with_dequantized_matmul(oracle):
    w = cases.std_weights(64, 2048, 5)
    x = cases.std_weights(1, 2048, 6)[0]
    blocks = oracle.quantize_q4_0(w)
    xq, xd = oracle.quantize_q8_0(x)
    y = oracle.gemv_q4_0(blocks, 2048, xq, xd)
    x_deq = xq.astype(np.float32) * np.repeat(xd.astype(np.float32), 32)
    ref = oracle.dequantize_q4_0(blocks, 2048).astype(np.float64) @ x_deq.astype(np.float64)
    np.testing.assert_allclose(y, ref, rtol=1e-4, atol=1e-3)


def test_gemv_rejects_wrong_dtypes_and_ragged_lanes(oracle):
    blocks = oracle.quantize_q4_0(cases.std_weights(2, 256, 11))
    xq, xd = oracle.quantize_q8_0(cases.std_weights(1, 256, 12)[0])
    assert oracle.gemv_q4_0(blocks, 256, xq, xd).dtype == np.float32
    with pytest.raises(TypeError):
        oracle.gemv_q4_0(blocks, 256, xq.astype(np.int32), xd)
    with pytest.raises(ValueError):
        oracle.gemv_q4_0(oracle.quantize_q4_0(cases.std_weights(2, 128, 13)), 128,
                         *oracle.quantize_q8_0(cases.std_weights(1, 128, 14)[0]))


def test_engine_x_layout(oracle):
    xq, xd = oracle.quantize_q8_0(cases.std_weights(1, 64, 15)[0])
    packed = oracle.pack_x_for_engine(xq, xd)
    assert packed.dtype == np.uint8 and packed.shape == (64 + 2 * 4,)
    assert np.array_equal(packed[:64].view(np.int8), xq)
    assert np.array_equal(packed[64:].view(np.float32), xd.astype(np.float32))


def test_thread_count_does_not_change_bits(oracle):
    blocks = oracle.quantize_q4_0(cases.std_weights(333, 1024, 21))
    xq, xd = oracle.quantize_q8_0(cases.std_weights(1, 1024, 22)[0])
    a = oracle.gemv_q4_0(blocks, 1024, xq, xd, threads=1)
    b = oracle.gemv_q4_0(blocks, 1024, xq, xd, threads=7)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


# --------------------------------------------- BASELINE configs 0 and 1

def test_config0_single_gemv(oracle, golden):
    rec = golden["config0"]
    blocks = oracle.quantize_q4_0(cases.shape_weights(rec["n"], rec["k"], rec["seed"]))
    assert cases.sha256(blocks) == rec["sha256_blocks"]
    y = oracle.gemv_q4_0_f32(blocks, rec["k"], cases.shape_x(rec["k"], rec["seed"]))
    assert np.array_equal(y.view(np.uint32), _y(rec["y"]).view(np.uint32))


@pytest.mark.parametrize("name,n,k,seed", [s for s in cases.LLAMA_1B_SHAPES if s[0] != "lm_head"])
def test_llama_1b_shapes_and_ksplit(oracle, golden, name, n, k, seed):
    rec = golden["shapes"][name]
    blocks = oracle.quantize_q4_0(cases.shape_weights(n, k, seed))
    x = cases.shape_x(k, seed)
    assert cases.sha256(blocks) == rec["sha256_blocks"]
    y = oracle.gemv_q4_0_f32(blocks, k, x)
    assert cases.sha256(y) == rec["sha256_y"]
    for parts in cases.SPLITS:
        if name in cases.K_SPLIT:
            kk = k // parts
            partials = [oracle.gemv_q4_0_f32(cases.k_slice_blocks(blocks, k, r, parts), kk, x[r * kk:(r + 1) * kk])
                        for r in range(parts)]
            assert cases.sha256(oracle.allreduce_ordered(partials)) == rec[f"sha256_ksplit{parts}"]
        else:
            # row split: each rank's rows are an independent GEMV over the full x
            rows = n // parts
            ys = [oracle.gemv_q4_0_f32(blocks[r * rows:(r + 1) * rows], k, x) for r in range(parts)]
            assert cases.sha256(np.concatenate(ys)) == rec["sha256_y"]


def test_allreduce_order_is_rank_order(oracle):
    a = np.array([1e8, 1.0, -1.0], dtype=np.float32)
    b = np.array([1.0, 1e8, 1e8], dtype=np.float32)
    c = np.array([-1e8, -1e8, -1e8], dtype=np.float32)
    got = oracle.allreduce_ordered([a, b, c])
    want = (a + b) + c
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert not np.array_equal(got, (a + c) + b)   # the order is observable


def test_gemv2_chunk_offset_is_a_bijection(oracle):
    rows, k = 64, 1024
    nch, row_bytes = k // 256, k // 32 * 18
    seen = {p: set() for p in range(4)}
    for r in range(rows):
        for c in range(nch):
            off, port = oracle.gemv2_chunk_offset(r, c, rows, k)
            assert port == r // (rows // 4) and off % 144 == 0
            seen[port].add(off)
    for p in range(4):
        assert sorted(seen[p]) == list(range(0, rows // 4 * row_bytes, 144))


def test_ragged_lane_rule_equals_zero_padding(oracle):
    """The 3B model's attn_output shard at 8 ranks has 12 blocks per row (a
    multiple of 8 is what q4_0.py:166-167 asks). The lane rule b mod 8 applied
    to 12 blocks gives the same bits as padding every row with zero blocks to
    16 and x with zeros: what the GPU decoder does with that shard."""
    w = cases.std_weights(64, 384, 31)
    x = cases.std_weights(1, 384, 32)[0] * 3
    blocks = oracle.quantize_q4_0(w)
    xq, xd = oracle.quantize_q8_0(x)
    ragged = oracle.gemv_q4_0(blocks, 384, xq, xd, allow_ragged_lanes=True)
    pb = np.zeros((64, 512 // 32 * 18), np.uint8)
    pb[:, : 384 // 32 * 18] = blocks
    xp = np.zeros(512, np.float32)
    xp[:384] = x
    xq2, xd2 = oracle.quantize_q8_0(xp)
    padded = oracle.gemv_q4_0(pb, 512, xq2, xd2)
    assert np.array_equal(ragged.view(np.uint32), padded.view(np.uint32))
    # and the lane rule itself, restated: lane b % 8 sums its blocks in order
    qs, ds = oracle.unpack_q4_0(blocks, 384)
    for r in (0, 17, 63):
        lanes = np.zeros(8, np.float32)
        for b in range(12):
            s = int(np.dot(qs[r, 32 * b:32 * b + 32].astype(np.int64), xq[32 * b:32 * b + 32].astype(np.int64)))
            t = np.float32(np.float32(s) * np.float32(ds[r, b])) * np.float32(xd[b])
            lanes[b % 8] = np.float32(lanes[b % 8] + t)
        assert np.float32(oracle.tree_sum(lanes)).view(np.uint32) == ragged[r].view(np.uint32)


def test_decode_oracle_runs_3b_width_at_8_ranks(oracle, pkg):
    from llm_kv260_b200 import model
    hp = dict(cases.W3B, n_layer=1, n_vocab=256)
    m = model.synth_model(hp, seed=9)
    d8 = oracle.Decoder(m, nranks=8, ctx_max=8)
    tok, val = d8.forward(3, 0)
    assert 0 <= tok < 256 and np.isfinite(val)
    d8.close()
