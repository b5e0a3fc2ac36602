"""The decode oracle pinned to the reference runtime's own code.

oracle/_ref compiles board/tp/tp_llama.cpp's model, engine, ops, forward and
sample_token sections on this host (oracle/ref_runtime.cpp, oracle/refshim/).
tests/golden/ref_decode.json holds what that code computed for the seeded
models of cases.REF_DECODE_CASES (gen_ref_decode.py), so the oracle is checked
against it everywhere; where oracle/_ref is built (the reference checkout is
present), the ops are also compared call by call on fresh random inputs."""

from __future__ import annotations

import json
import os

import numpy as np
import pytest

import cases

GOLDEN = os.path.dirname(os.path.abspath(cases.__file__))


@pytest.fixture(scope="module")
def ref_decode() -> dict:
    with open(os.path.join(GOLDEN, "ref_decode.json")) as fh:
        return json.load(fh)["cases"]


@pytest.fixture(scope="module")
def ref(oracle):
    if not oracle.ref_available() and not oracle.build_ref(oracle.default_reference_root()):
        pytest.skip("oracle/_ref needs the reference checkout; the fixture tests still pin the oracle")
    return oracle.ref_lib()


def bits(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def p(a: np.ndarray) -> int:
    return a.ctypes.data


@pytest.mark.parametrize("name", sorted(cases.REF_DECODE_CASES))
def test_oracle_reproduces_reference_runtime(oracle, ref_decode, name):
    """Every token, logit value and residual digest the reference runtime made,
    position by position, and each rank's last logits."""
    hp, _, ranks, n_prompt, n_pos, _, _ = cases.REF_DECODE_CASES[name]
    want = ref_decode[name]
    m, prompt = cases.ref_decode_model(name)
    assert [int(x) for x in prompt] == want["prompt"]
    dec = oracle.Decoder(m, nranks=ranks, ctx_max=n_pos, kv_f16=False, round_mode=oracle.ROUND_ROUNDF)
    tok = None
    for i in range(n_pos):
        inp = int(prompt[i]) if i < n_prompt else tok
        tok, val = dec.forward(inp, i)
        assert tok == want["tokens"][i], f"token at position {i}"
        assert int(np.float32(val).view(np.uint32)) == want["value_bits"][i], f"logit at position {i}"
        assert cases.sha256(dec.residual()) == want["residual_sha256"][i], f"residual at position {i}"
    for r in range(ranks):
        assert cases.sha256(dec.logits(r)) == want["last_logits_sha256"][r], f"rank {r} logits"
    dec.close()


def test_v_expf_matches_reference(oracle, ref):
    rng = np.random.default_rng(1)
    x = np.concatenate([rng.uniform(-110.0, 110.0, 200000), rng.standard_normal(100000) * 3,
                        np.array([0.0, -0.0, 88.7, 88.8, -87.3, -103.9, -104.0, 126.0, -126.0, 200.0, -200.0,
                                  np.inf, -np.inf], np.float64)]).astype(np.float32)
    x = np.concatenate([x, np.zeros((-len(x)) % 4, np.float32)])
    want = np.empty_like(x)
    for i in range(0, len(x), 4):
        ref.ref_v_expf4(p(x[i:i + 4]), p(want[i:i + 4]))
    got = np.array([oracle.v_expf(float(v)) for v in x[:20000]], np.float32)
    assert np.array_equal(bits(got), bits(want[:20000]))
    lib = oracle.lib()
    got_all = np.array([lib.odec_v_expf(float(v)) for v in x], np.float32)
    assert np.array_equal(bits(got_all), bits(want))


@pytest.mark.parametrize("n", [256, 2048, 3072, 8192])
def test_rmsnorm_matches_reference(oracle, ref, n):
    rng = np.random.default_rng(n)
    for scale in (1e-3, 1.0, 30.0):
        x = (rng.standard_normal(n) * scale).astype(np.float32)
        w = (1 + 0.05 * rng.standard_normal(n)).astype(np.float32)
        want = np.empty(n, np.float32)
        ref.ref_rmsnorm(p(want), p(x), p(w), n, 1e-5)
        assert np.array_equal(bits(oracle.rmsnorm(x, w, 1e-5)), bits(want))


@pytest.mark.parametrize("d", [64, 128])
def test_rope_matches_reference(oracle, ref, d):
    rng = np.random.default_rng(d)
    for pos in (0, 1, 17, 423, 4351):
        cs = np.empty(d, np.float32)
        ref.ref_rope_table(p(cs), d, pos, 500000.0)
        assert np.array_equal(bits(oracle.rope_table(d, pos, 500000.0)), bits(cs))
        x = rng.standard_normal(4 * d).astype(np.float32)
        want = x.copy()
        ref.ref_rope(p(want), 4, d, p(cs))
        assert np.array_equal(bits(oracle.rope(x, 4, d, cs)), bits(want))


def test_embed_and_silu_match_reference(oracle, ref, pkg):
    from llm_kv260_b200 import model
    rng = np.random.default_rng(3)
    te = model.q4_0_rows(rng, 64, 2048)
    for tok in (0, 5, 63):
        want = np.empty(2048, np.float32)
        ref.ref_embed(p(want), p(te), tok, 2048)
        assert np.array_equal(bits(oracle.embed(te, tok, 2048)), bits(want))
    g = (rng.standard_normal(8192) * 4).astype(np.float32)
    u = rng.standard_normal(8192).astype(np.float32)
    want = np.empty(8192, np.float32)
    ref.ref_silu_mul(p(want), p(g), p(u), 8192)
    assert np.array_equal(bits(oracle.silu_mul(g, u)), bits(want))


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("B", [1, 2, 3, 4])
def test_attention_matches_reference(oracle, ref, d, B):
    """attention_heads over a float32 cache (the reference's), positions
    across 4-lane tails."""
    rng = np.random.default_rng(10 * d + B)
    ctx = 310
    kc = rng.standard_normal((ctx, d)).astype(np.float32)
    vc = rng.standard_normal((ctx, d)).astype(np.float32)
    q = (rng.standard_normal(B * d) * 0.3).astype(np.float32)
    scale = np.float32(1.0 / np.sqrt(np.float32(d)))
    lib = oracle.lib()
    for pos in (0, 3, 4, 129, 290, 309):
        sc = np.zeros(4 * ctx, np.float32)
        want = np.empty(B * d, np.float32)
        ref.ref_attention_heads(B, p(q), p(kc), p(vc), d, pos, d, float(scale), p(sc), ctx, p(want))
        sc2 = np.zeros(4 * ctx, np.float32)
        got = np.empty(B * d, np.float32)
        lib.odec_attention(B, p(q), p(kc), p(vc), 0, d, pos, d, float(scale), p(sc2), ctx, p(got))
        assert np.array_equal(bits(got), bits(want)), pos


def test_quantize_x_matches_reference_roundf(oracle, ref, golden):
    """engine_t::quantize_x (roundf, tp_llama.cpp:330-352) against the oracle's
    runtime rounding on random vectors and the rounding edges."""
    rng = np.random.default_rng(5)
    xs = [rng.standard_normal(4096).astype(np.float32) * s for s in (1e-4, 1.0, 300.0)]
    edge = np.zeros(64, np.float32)
    edge[0] = 127.0
    edge[1:9] = np.array([0.49999997, 0.5, 1.5, 2.5, -0.5, -2.5, 126.5, -126.5], np.float32)
    edge[32] = 127.0
    edge[33] = -0.0
    xs.append(edge)
    for x in xs:
        k = x.shape[0]
        qs = np.empty(k, np.int8)
        xd = np.empty(k // 32, np.float32)
        ref.ref_quantize_x(p(x), p(qs), p(xd), k)
        oq, od = oracle.quantize_q8_0(x, round_mode=oracle.ROUND_ROUNDF)
        assert np.array_equal(oq, qs)
        assert np.array_equal(bits(od.astype(np.float32)), bits(xd))


@pytest.mark.parametrize("ranks,gemv2", [(1, False), (2, True), (4, False)])
def test_reference_runtime_live_against_oracle(oracle, ref, pkg, tmp_path, ranks, gemv2):
    """A model no fixture holds: the reference runtime and the oracle side by
    side, every position."""
    from gguf_model import write_gguf
    from llm_kv260_b200 import model
    hp = dict(cases.TPW, n_layer=1)
    m = model.synth_model(hp, seed=77)
    prompt = model.random_prompt(4, hp["n_vocab"], seed=78)
    path = write_gguf(m, str(tmp_path / "m.gguf"))
    rr = oracle.RefRuntime(path, nranks=ranks, ctx_max=16, gemv2=gemv2)
    od = oracle.Decoder(m, nranks=ranks, ctx_max=16, kv_f16=False, round_mode=oracle.ROUND_ROUNDF)
    tok = None
    for i in range(16):
        inp = int(prompt[i]) if i < 4 else tok
        tr, vr = rr.forward(inp, i)
        to, vo = od.forward(inp, i)
        assert (tr, np.float32(vr).view(np.uint32)) == (to, np.float32(vo).view(np.uint32)), i
        assert np.array_equal(bits(rr.read(0, hp["n_embd"])), bits(od.residual())), i
        tok = to
    rr.close()
    od.close()
