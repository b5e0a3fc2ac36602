"""The decode-step oracle (oracle/decode_oracle.c) on the CPU: each op against
an independent statement of the same arithmetic, and the decode loop's
bookkeeping. The reference runtime itself cannot run here (NEON, libllama),
so these pin the restatement to its own definitions, not to the reference."""

from __future__ import annotations

import math

import numpy as np
import pytest

TINY = dict(n_layer=2, n_embd=512, n_ff=1024, n_head=8, n_head_kv=2, head_dim=64, n_vocab=1024,
            rope_base=500000.0, rms_eps=1e-5)


def f32(x) -> np.float32:
    return np.float32(x)


def test_v_expf_is_exp_within_two_ulps(oracle):
    xs = np.concatenate([np.linspace(-87.0, 88.0, 40001, dtype=np.float32),
                         np.float32([0.0, -0.0, 1e-30, -1e-30, 0.5, -0.5])])
    for x in xs:
        got = np.float32(oracle.v_expf(float(x)))
        want = math.exp(float(x))
        ulp = float(np.spacing(np.float32(want)))
        assert abs(float(got) - want) <= 2 * ulp, (x, got, want)


def test_v_expf_special_ranges(oracle):
    assert oracle.v_expf(0.0) == 1.0
    assert oracle.v_expf(-200.0) == 0.0              # |n| > 192: the underflow branch
    assert 0.0 < oracle.v_expf(-100.0) < 1e-40        # the subnormal branch (126 < |n| <= 192)
    assert math.isinf(oracle.v_expf(200.0))


def test_rmsnorm_is_the_four_lane_double_sum(oracle):
    rng = np.random.default_rng(3)
    for n in (4, 64, 2048, 3072):
        x = (rng.standard_normal(n) * rng.choice([1e-3, 1.0, 50.0], n)).astype(np.float32)
        w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
        lanes = [0.0, 0.0, 0.0, 0.0]
        for i in range(n):                          # python floats are doubles: sequential per lane
            lanes[i % 4] += float(x[i]) * float(x[i])
        ss = (lanes[0] + lanes[2]) + (lanes[1] + lanes[3])
        scale = f32(1.0) / np.sqrt(f32(np.float32(ss / n) + f32(1e-5)), dtype=np.float32)
        want = (x * scale) * w
        got = oracle.rmsnorm(x, w, 1e-5)
        assert np.array_equal(got.view(np.uint32), want.astype(np.float32).view(np.uint32)), n


def test_rope_pairs(oracle):
    rng = np.random.default_rng(4)
    d, heads = 64, 3
    x = rng.standard_normal(heads * d).astype(np.float32)
    cs = oracle.rope_table(d, 17, 500000.0)
    got = oracle.rope(x, heads, d, cs)
    want = x.copy()
    for h in range(heads):
        for i in range(d // 2):
            c, s = cs[2 * i], cs[2 * i + 1]
            x0, x1 = x[h * d + 2 * i], x[h * d + 2 * i + 1]
            want[h * d + 2 * i] = x0 * c - x1 * s
            want[h * d + 2 * i + 1] = x0 * s + x1 * c
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert np.array_equal(oracle.rope_table(d, 0, 500000.0), np.tile(np.float32([1.0, 0.0]), d // 2))


def test_rope_table_of_the_library_is_the_oracles(pkg, oracle):
    """The decoder uploads a host-computed table; it must be the oracle's bits."""
    from llm_kv260_b200 import decoder
    for d in (64, 128):
        for pos in (0, 1, 7, 23, 400, 4351):
            a = decoder.rope_table(d, pos, 500000.0)
            b = oracle.rope_table(d, pos, 500000.0)
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), (d, pos)


def test_embed_is_the_dequantised_row(oracle):
    from llm_kv260_b200 import model
    rng = np.random.default_rng(5)
    te = model.q4_0_rows(rng, 40, 256)
    deq = oracle.dequantize_q4_0(te, 256)
    for tok in (0, 13, 39):
        assert np.array_equal(oracle.embed(te, tok, 256), deq[tok])


def test_silu_mul_close_to_the_formula(oracle):
    g = np.linspace(-20, 20, 4001, dtype=np.float32)
    u = np.float32(1.5) * np.ones_like(g)
    got = oracle.silu_mul(g, u)
    want = g.astype(np.float64) / (1 + np.exp(-g.astype(np.float64))) * 1.5
    assert np.allclose(got, want, rtol=3e-7, atol=1e-30)


def test_attention_close_to_softmax_attention(oracle):
    rng = np.random.default_rng(6)
    B, d, n = 4, 64, 37
    q = rng.standard_normal((B, d)).astype(np.float32)
    k = rng.standard_normal((n, d)).astype(np.float32)
    v = rng.standard_normal((n, d)).astype(np.float32)
    scale = 1 / math.sqrt(d)
    for kv in (np.float32, np.float16):
        kc, vc = k.astype(kv), v.astype(kv)
        got = oracle.attention(q, kc, vc, n - 1, scale)
        s = q.astype(np.float64) @ kc.astype(np.float64).T * scale
        p = np.exp(s - s.max(axis=1, keepdims=True))
        want = (p / p.sum(axis=1, keepdims=True)) @ vc.astype(np.float64)
        assert np.allclose(got, want, rtol=1e-4, atol=1e-5)


@pytest.fixture(scope="module")
def tiny_model():
    from llm_kv260_b200 import model
    return model.synth_model(TINY, seed=11)


def test_generate_is_forward_then_pick(oracle, tiny_model):
    from llm_kv260_b200 import model
    prompt = model.random_prompt(6, TINY["n_vocab"], seed=1)
    a = oracle.Decoder(tiny_model, nranks=1, ctx_max=32)
    toks = a.generate(prompt, 8)
    b = oracle.Decoder(tiny_model, nranks=1, ctx_max=32)
    t = None
    for i, p in enumerate(prompt):
        t, _ = b.forward(int(p), i)
    seq = [t]
    for i in range(7):
        t, _ = b.forward(t, len(prompt) + i)
        seq.append(t)
    assert list(toks) == seq
    assert np.array_equal(a.residual(), b.residual())
    # the pick is the first index of the largest logit
    lg = b.logits()
    assert seq[-1] == int(np.argmax(lg))


def test_tensor_parallel_simulation_stays_close_to_one_rank(oracle, tiny_model):
    """K-split partials summed in rank order change low bits only."""
    prompt = [3, 141, 59, 265]
    logits = {}
    for n in (1, 2):
        dec = oracle.Decoder(tiny_model, nranks=n, ctx_max=16, kv_f16=False)
        for i, p in enumerate(prompt):
            dec.forward(p, i)
        logits[n] = np.concatenate([dec.logits(r) for r in range(n)])
    assert np.allclose(logits[1], logits[2], rtol=1e-3, atol=1e-3)


def test_decoder_rejects_bad_shapes(oracle, tiny_model):
    bad = dict(tiny_model)
    bad["n_head_kv"] = 3      # 8 heads do not group over 3 KV heads
    with pytest.raises(ValueError):
        oracle.Decoder(bad, nranks=1)
