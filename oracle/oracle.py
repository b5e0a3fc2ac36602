"""CPU oracle, Python face. TEST INFRASTRUCTURE ONLY.

The parity tests, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` call this as the checker. The product (the CUDA library under
``llm-kv260_b200/``) never imports it.

The functions mirror the reference contract ``src/llm_kv260/q4_0.py`` name for
name, with the same argument meaning and the same errors (TypeError for a wrong
dtype, ValueError for a wrong shape), and run the C restatement in
``q4_0_oracle.c`` through ctypes. The rank-ordered sum restates
``board/tp/tp_llama.cpp:515-521``.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

QK = 32            # q4_0.py:59
Q4_0_BYTES = 18    # q4_0.py:60
Q8_0_BYTES = 34    # q4_0.py:61
LANES = 8          # q4_0.py:62
CONTRACT_VERSION = "llm-kv260/w4a8-q4_0-v2"   # q4_0.py:64

ROUND_CONTRACT = 0   # floor(|s| + 0.5f) with sign, q4_0.py:96
ROUND_ROUNDF = 1     # roundf, tp_llama.cpp:343 (vcvtaq)

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle_q4.so")
_lib = None


def build(force: bool = False) -> str:
    """Compile the C restatement with its Makefile (gcc, -ffp-contract=off)."""
    srcs = [os.path.join(_HERE, f) for f in ("q4_0_oracle.c", "q4_0_oracle.h", "decode_oracle.c", "decode_oracle.h")]
    newest = max(os.path.getmtime(f) for f in srcs)
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < newest:
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P, I64, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        sig = {
            "oracle_f32_to_f16": (ctypes.c_uint16, [ctypes.c_float]),
            "oracle_f16_to_f32": (ctypes.c_float, [ctypes.c_uint16]),
            "oracle_tree_sum8": (ctypes.c_float, [P]),
            "oracle_quantize_q8_0": (I, [P, I64, P, P, I]),
            "oracle_quantize_q4_0": (I, [P, I64, I64, P, I]),
            "oracle_unpack_q4_0": (I, [P, I64, I64, P, P]),
            "oracle_dequantize_q4_0": (I, [P, I64, I64, P]),
            "oracle_gemv_q4_0": (I, [P, I64, I64, P, P, P, I, I]),
            "oracle_gemv_q4_0_f32": (I, [P, I64, I64, P, P, I, I]),
            "oracle_pack_x_for_engine": (I, [P, P, I64, P]),
            "oracle_gemv_q4_0_packed": (I, [P, I64, I64, P, P, I]),
            "oracle_gemv2_chunk_offset": (I64, [I, I, I, I, ctypes.POINTER(ctypes.c_int)]),
            "oracle_allreduce_ordered": (I, [P, I, I64, P]),
            "odec_v_expf": (ctypes.c_float, [ctypes.c_float]),
            "odec_rmsnorm": (None, [P, P, P, I, ctypes.c_float]),
            "odec_rope_table": (None, [P, I, I, ctypes.c_float]),
            "odec_rope_table_freqs": (None, [P, I, I, ctypes.c_float, P]),
            "odec_set_rope_freqs": (I, [P, P]),
            "odec_rope": (None, [P, I, I, P]),
            "odec_silu_mul": (None, [P, P, P, I]),
            "odec_embed": (None, [P, P, I, I]),
            "odec_attention": (None, [I, P, P, P, I, I64, I, I, ctypes.c_float, P, I, P]),
            "odec_create": (I, [P, P, P, P, P]),
            "odec_destroy": (None, [P]),
            "odec_forward": (I, [P, I, I, P, P]),
            "odec_generate": (I, [P, P, I, I, P]),
            "odec_read": (I, [P, I, I, P, I64]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def _check(rc: int, what: str) -> None:
    if rc == -1:
        raise ValueError(f"{what}: shape rejected by the contract")
    if rc != 0:
        raise RuntimeError(f"{what}: oracle returned {rc}")


def default_threads() -> int:
    return max(1, len(os.sched_getaffinity(0)))


# ------------------------------------------------------------- float16 / tree

def f32_to_f16_bits(v: float) -> int:
    return int(lib().oracle_f32_to_f16(ctypes.c_float(v)))


def f16_bits_to_f32(h: int) -> float:
    return float(lib().oracle_f16_to_f32(ctypes.c_uint16(h)))


def tree_sum(values: np.ndarray) -> np.ndarray:
    """q4_0.py:67-78 for the 8-lane case the contract uses (last axis 8)."""
    values = np.ascontiguousarray(values, dtype=np.float32)
    if values.shape[-1] != LANES:
        raise ValueError(f"the oracle's tree is over {LANES} lanes, got {values.shape[-1]}")
    flat = values.reshape(-1, LANES)
    out = np.empty(flat.shape[0], dtype=np.float32)
    for i in range(flat.shape[0]):
        out[i] = lib().oracle_tree_sum8(_ptr(np.ascontiguousarray(flat[i])))
    return out.reshape(values.shape[:-1])


# ------------------------------------------------------------------ quantizers

def quantize_q8_0(x: np.ndarray, round_mode: int = ROUND_CONTRACT) -> tuple[np.ndarray, np.ndarray]:
    """q4_0.py:83-97. Returns (q int8 [K], d float16 [K/32])."""
    if x.dtype != np.float32:
        raise TypeError(f"activations must be float32, got {x.dtype}")
    if x.ndim != 1 or x.shape[0] % QK:
        raise ValueError(f"x must be 1-D with a multiple of {QK} elements, got {x.shape}")
    x = np.ascontiguousarray(x)
    q = np.empty(x.shape[0], dtype=np.int8)
    d = np.empty(x.shape[0] // QK, dtype=np.uint16)
    _check(lib().oracle_quantize_q8_0(_ptr(x), x.shape[0], _ptr(q), _ptr(d), round_mode), "quantize_q8_0")
    return q, d.view(np.float16)


def quantize_q4_0(w: np.ndarray, threads: int | None = None) -> np.ndarray:
    """q4_0.py:100-121. Returns uint8 [N, K/32*18]."""
    if w.dtype != np.float32:
        raise TypeError(f"weights must be float32, got {w.dtype}")
    n, k = w.shape
    if k % QK:
        raise ValueError(f"in_features must be a multiple of {QK}, got {k}")
    w = np.ascontiguousarray(w)
    out = np.empty((n, k // QK * Q4_0_BYTES), dtype=np.uint8)
    _check(lib().oracle_quantize_q4_0(_ptr(w), n, k, _ptr(out), threads or default_threads()), "quantize_q4_0")
    return out


# ----------------------------------------------------------------------- codec

def unpack_q4_0(blocks: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray]:
    """q4_0.py:126-140."""
    if blocks.dtype != np.uint8:
        raise TypeError(f"expected uint8 block bytes, got {blocks.dtype}")
    n = blocks.shape[0]
    nb = k // QK
    if blocks.shape[1] != nb * Q4_0_BYTES:
        raise ValueError(f"{blocks.shape[1]} bytes per row is not {nb} blocks of {Q4_0_BYTES}")
    blocks = np.ascontiguousarray(blocks)
    ints = np.empty((n, k), dtype=np.int8)
    d = np.empty((n, nb), dtype=np.uint16)
    _check(lib().oracle_unpack_q4_0(_ptr(blocks), n, k, _ptr(ints), _ptr(d)), "unpack_q4_0")
    return ints, d.view(np.float16)


def dequantize_q4_0(blocks: np.ndarray, k: int) -> np.ndarray:
    """q4_0.py:143-146."""
    if blocks.dtype != np.uint8:
        raise TypeError(f"expected uint8 block bytes, got {blocks.dtype}")
    n = blocks.shape[0]
    if blocks.shape[1] != k // QK * Q4_0_BYTES:
        raise ValueError("row byte count does not match k")
    blocks = np.ascontiguousarray(blocks)
    out = np.empty((n, k), dtype=np.float32)
    _check(lib().oracle_dequantize_q4_0(_ptr(blocks), n, k, _ptr(out)), "dequantize_q4_0")
    return out


# ------------------------------------------------------------------------ gemv

def gemv_q4_0(blocks: np.ndarray, k: int, xq: np.ndarray, xd: np.ndarray,
              threads: int | None = None, allow_ragged_lanes: bool = False) -> np.ndarray:
    """q4_0.py:151-182: float32 [N] in the engine's order."""
    if xq.dtype != np.int8 or xd.dtype != np.float16:
        raise TypeError(f"x must be (int8, float16), got ({xq.dtype}, {xd.dtype})")
    if blocks.dtype != np.uint8:
        raise TypeError(f"expected uint8 block bytes, got {blocks.dtype}")
    n = blocks.shape[0]
    nb = k // QK
    if k % QK or blocks.shape[1] != nb * Q4_0_BYTES:
        raise ValueError(f"{blocks.shape[1]} bytes per row is not {nb} blocks of {Q4_0_BYTES}")
    if xq.shape != (k,) or xd.shape != (nb,):
        raise ValueError(f"x shapes {xq.shape}, {xd.shape} do not match K={k}")
    if nb % LANES and not allow_ragged_lanes:
        raise ValueError(f"{nb} blocks is not a multiple of {LANES} lanes")
    blocks = np.ascontiguousarray(blocks)
    xq = np.ascontiguousarray(xq)
    xd16 = np.ascontiguousarray(xd).view(np.uint16)
    y = np.empty(n, dtype=np.float32)
    _check(lib().oracle_gemv_q4_0(_ptr(blocks), n, k, _ptr(xq), _ptr(xd16), _ptr(y),
                                  threads or default_threads(), int(allow_ragged_lanes)), "gemv_q4_0")
    return y


def gemv_q4_0_f32(blocks: np.ndarray, k: int, x: np.ndarray, threads: int | None = None,
                  round_mode: int = ROUND_CONTRACT) -> np.ndarray:
    """q4_0.py:185-188."""
    xq, xd = quantize_q8_0(x, round_mode)
    return gemv_q4_0(blocks, k, xq, xd, threads)


def pack_x_for_engine(xq: np.ndarray, xd: np.ndarray) -> np.ndarray:
    """q4_0.py:193-200: int8[K] then float32[K/32]."""
    k = xq.shape[0]
    out = np.empty(k + 4 * (k // QK), dtype=np.uint8)
    _check(lib().oracle_pack_x_for_engine(_ptr(np.ascontiguousarray(xq)),
                                          _ptr(np.ascontiguousarray(xd).view(np.uint16)), k, _ptr(out)),
           "pack_x_for_engine")
    return out


def gemv_q4_0_packed(blocks: np.ndarray, k: int, xpacked: np.ndarray, threads: int | None = None) -> np.ndarray:
    """The GEMV over the engine's activation buffer (board/kv260gemv/gemv_dev.h:19-23)."""
    n = blocks.shape[0]
    if xpacked.dtype != np.uint8 or xpacked.shape != (k + 4 * (k // QK),):
        raise ValueError("xpacked must be uint8[k + 4*k/32]")
    y = np.empty(n, dtype=np.float32)
    _check(lib().oracle_gemv_q4_0_packed(_ptr(np.ascontiguousarray(blocks)), n, k,
                                         _ptr(np.ascontiguousarray(xpacked)), _ptr(y),
                                         threads or default_threads()), "gemv_q4_0_packed")
    return y


def gemv2_chunk_offset(r: int, c: int, rows: int, k: int) -> tuple[int, int]:
    """board/kv260gemv/gemv2_dev.h:66-72. Returns (byte offset, port)."""
    port = ctypes.c_int(0)
    off = lib().oracle_gemv2_chunk_offset(r, c, rows, k, ctypes.byref(port))
    return int(off), int(port.value)


def allreduce_ordered(partials: list[np.ndarray]) -> np.ndarray:
    """tp_llama.cpp:515-521: p0 + p1 + ... + p{n-1}, left to right, per element."""
    parts = [np.ascontiguousarray(p, dtype=np.float32) for p in partials]
    n = len(parts)
    length = parts[0].shape[0]
    if any(p.shape != (length,) for p in parts):
        raise ValueError("partials must share one 1-D shape")
    ptrs = (ctypes.c_void_p * n)(*[_ptr(p) for p in parts])
    out = np.empty(length, dtype=np.float32)
    _check(lib().oracle_allreduce_ordered(ctypes.cast(ptrs, ctypes.c_void_p), n, length, _ptr(out)),
           "allreduce_ordered")
    return out


# ------------------------------------------------------------------ decode step
# decode_oracle.c: runtime::forward of board/tp/tp_llama.cpp (822-883) and its
# ops, restated per NEON lane; parity with the reference itself is unpinned.

def v_expf(x: float) -> float:
    """tp_llama.cpp:530-553 (one lane)."""
    return float(lib().odec_v_expf(float(x)))


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """tp_llama.cpp:557-569."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    if x.shape != w.shape or x.ndim != 1 or x.shape[0] % 4:
        raise ValueError("x and w must be 1-D of one length, a multiple of 4")
    out = np.empty_like(x)
    lib().odec_rmsnorm(_ptr(out), _ptr(x), _ptr(w), x.shape[0], eps)
    return out


def rope_table_freqs(d: int, pos: int, base: float, freqs: np.ndarray) -> np.ndarray:
    """tp_llama.cpp:574-580 with the model's frequency factors."""
    cs = np.empty(d, dtype=np.float32)
    f = np.ascontiguousarray(freqs, dtype=np.float32)
    lib().odec_rope_table_freqs(_ptr(cs), d, pos, base, _ptr(f))
    return cs


def rope_table(d: int, pos: int, base: float) -> np.ndarray:
    """tp_llama.cpp:574-580 without freq factors: cos, sin interleaved, d floats."""
    cs = np.empty(d, dtype=np.float32)
    lib().odec_rope_table(_ptr(cs), d, pos, base)
    return cs


def rope(x: np.ndarray, n_heads: int, d: int, cs: np.ndarray) -> np.ndarray:
    """tp_llama.cpp:581-591, on a copy."""
    y = np.array(x, dtype=np.float32, copy=True)
    cs = np.ascontiguousarray(cs, dtype=np.float32)
    lib().odec_rope(_ptr(y), n_heads, d, _ptr(cs))
    return y


def silu_mul(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """tp_llama.cpp:615-622."""
    g = np.ascontiguousarray(gate, dtype=np.float32)
    u = np.ascontiguousarray(up, dtype=np.float32)
    out = np.empty_like(g)
    lib().odec_silu_mul(_ptr(out), _ptr(g), _ptr(u), g.shape[0])
    return out


def embed(token_embd: np.ndarray, token: int, n_embd: int) -> np.ndarray:
    """tp_llama.cpp:593-604."""
    t = np.ascontiguousarray(token_embd, dtype=np.uint8)
    out = np.empty(n_embd, dtype=np.float32)
    lib().odec_embed(_ptr(out), _ptr(t), token, n_embd)
    return out


def attention(q: np.ndarray, kc: np.ndarray, vc: np.ndarray, pos: int, scale: float) -> np.ndarray:
    """attention_group (tp_llama.cpp:644-690): q [B, d] float32; kc, vc
    [>= pos+1, d] float32 or float16 (their bits used as stored)."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    B, d = q.shape
    f16 = kc.dtype == np.float16
    kc = np.ascontiguousarray(kc)
    vc = np.ascontiguousarray(vc)
    sc = np.empty((B, pos + 1), dtype=np.float32)
    out = np.empty((B, d), dtype=np.float32)
    lib().odec_attention(B, _ptr(q), _ptr(kc), _ptr(vc), int(f16), d, pos, d, scale, _ptr(sc), pos + 1, _ptr(out))
    return out


class _Config(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("n_layer", "n_embd", "n_ff", "n_head", "n_head_kv", "head_dim",
                                            "n_vocab")] + \
               [("rope_base", ctypes.c_float), ("rms_eps", ctypes.c_float)] + \
               [(n, ctypes.c_int) for n in ("ctx_max", "kv_f16", "nranks", "round_mode", "threads")]


class _Layer(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up",
                                               "ffn_down", "attn_norm", "ffn_norm")]


class Decoder:
    """The reference runtime's decode loop on the CPU, nranks shards simulated.

    `model` is a dict: hparams (n_layer, n_embd, n_ff, n_head, n_head_kv,
    head_dim, n_vocab, rope_base, rms_eps), "layers" (a list of dicts with
    attn_q, attn_k, attn_v, attn_output, ffn_gate, ffn_up, ffn_down as
    uint8 GGUF Q4_0 rows and attn_norm, ffn_norm as float32), "token_embd"
    and "output_norm"."""

    def __init__(self, model: dict, nranks: int = 1, ctx_max: int = 512, kv_f16: bool = True,
                 round_mode: int = ROUND_CONTRACT, threads: int | None = None):
        c = _Config()
        for n in ("n_layer", "n_embd", "n_ff", "n_head", "n_head_kv", "head_dim", "n_vocab"):
            setattr(c, n, int(model[n]))
        c.rope_base, c.rms_eps = float(model["rope_base"]), float(model["rms_eps"])
        c.ctx_max, c.kv_f16, c.nranks, c.round_mode = ctx_max, int(kv_f16), nranks, round_mode
        c.threads = threads or default_threads()
        self.n_vocab, self.n_embd, self.nranks = c.n_vocab, c.n_embd, nranks
        keep = []
        layers = (_Layer * c.n_layer)()
        for i, L in enumerate(model["layers"]):
            for n in _Layer._fields_:
                a = np.ascontiguousarray(L[n[0]])
                keep.append(a)
                setattr(layers[i], n[0], _ptr(a))
        te = np.ascontiguousarray(model["token_embd"], dtype=np.uint8)
        on = np.ascontiguousarray(model["output_norm"], dtype=np.float32)
        self._h = ctypes.c_void_p()
        _check(lib().odec_create(ctypes.byref(self._h), ctypes.byref(c), ctypes.cast(layers, ctypes.c_void_p),
                                 _ptr(te), _ptr(on)), "odec_create")
        if model.get("rope_freqs") is not None:
            rf = np.ascontiguousarray(model["rope_freqs"], dtype=np.float32)
            if rf.shape != (c.head_dim // 2,):
                raise ValueError(f"rope_freqs must hold head_dim/2 = {c.head_dim // 2} factors")
            _check(lib().odec_set_rope_freqs(self._h, _ptr(rf)), "odec_set_rope_freqs")

    def forward(self, token: int, pos: int) -> tuple[int, float]:
        t, v = ctypes.c_int(0), ctypes.c_float(0.0)
        _check(lib().odec_forward(self._h, token, pos, ctypes.byref(t), ctypes.byref(v)), "odec_forward")
        return int(t.value), float(v.value)

    def generate(self, prompt, n_gen: int) -> np.ndarray:
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(n_gen, dtype=np.int32)
        _check(lib().odec_generate(self._h, _ptr(p), p.shape[0], n_gen, _ptr(out)), "odec_generate")
        return out

    def residual(self) -> np.ndarray:
        out = np.empty(self.n_embd, dtype=np.float32)
        _check(lib().odec_read(self._h, 0, 0, _ptr(out), self.n_embd), "odec_read")
        return out

    def logits(self, rank: int = 0) -> np.ndarray:
        n = self.n_vocab // self.nranks
        out = np.empty(n, dtype=np.float32)
        _check(lib().odec_read(self._h, 1, rank, _ptr(out), n), "odec_read")
        return out

    def close(self) -> None:
        if self._h:
            lib().odec_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------- the reference's own runtime
# oracle/_ref/libref_runtime.so: board/tp/tp_llama.cpp's decode sections built
# on this host (ref_runtime.cpp, refshim/). It exists only where the reference
# checkout was present at build time; the golden fixtures it produced
# (tests/golden/ref_decode.json) carry its results everywhere else.

_REF_PATH = os.path.join(_HERE, "_ref", "libref_runtime.so")
_ref = None


def default_reference_root() -> str:
    """Where build() looks for the reference checkout: $LLM_KV260_REFERENCE,
    else a directory named "reference" beside this repository."""
    return os.environ.get("LLM_KV260_REFERENCE") or os.path.join(os.path.dirname(os.path.dirname(_HERE)), "reference")


def build_ref(reference_root: str, force: bool = False) -> str | None:
    """Build oracle/_ref from the reference checkout at `reference_root`
    (returns the library path), or None when the checkout is absent."""
    tp = os.path.join(reference_root, "board", "tp", "tp_llama.cpp")
    if not os.path.exists(tp):
        return None
    deps = [os.path.join(_HERE, f) for f in ("ref_runtime.cpp", "q4_0_oracle.c", "q4_0_oracle.h", "Makefile")]
    deps += [os.path.join(_HERE, "refshim", f) for f in os.listdir(os.path.join(_HERE, "refshim"))] + [tp]
    if force or not os.path.exists(_REF_PATH) or os.path.getmtime(_REF_PATH) < max(os.path.getmtime(f) for f in deps):
        subprocess.run(["make", "-s", "-C", _HERE, "ref", f"REF={os.path.abspath(reference_root)}"], check=True)
    return _REF_PATH


def ref_available() -> bool:
    return os.path.exists(_REF_PATH)


def ref_lib() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        if not os.path.exists(_REF_PATH):
            raise RuntimeError("oracle/_ref is not built (it needs the reference checkout)")
        L = ctypes.CDLL(_REF_PATH)
        P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        sig = {
            "ref_open": (I, [ctypes.c_char_p, I, I, I, I, ctypes.POINTER(P)]),
            "ref_forward": (I, [P, I, I, ctypes.POINTER(I), ctypes.POINTER(F)]),
            "ref_read": (I, [P, I, I, P, ctypes.c_int64]),
            "ref_close": (None, [P]),
            "ref_v_expf4": (None, [P, P]),
            "ref_rmsnorm": (None, [P, P, P, I, F]),
            "ref_rope_table": (None, [P, I, I, F]),
            "ref_rope": (None, [P, I, I, P]),
            "ref_embed": (None, [P, P, I, I]),
            "ref_silu_mul": (None, [P, P, P, I]),
            "ref_softmax_exp": (F, [P, I, F]),
            "ref_attention_heads": (None, [I, P, P, P, ctypes.c_int64, I, I, F, P, I, P]),
            "ref_quantize_x": (None, [P, P, P, I]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        _ref = L
    return _ref


class RefRuntime:
    """The reference runtime itself (runtime::init/forward/sample_token and
    load_model, tp_llama.cpp), `nranks` ranks as threads, reading a GGUF file.
    The engine is the FPGA's stand-in (the pinned q4_0 GEMV); float32 KV
    cache and the runtime's roundf quantiser, as on the boards."""

    def __init__(self, gguf_path: str, nranks: int = 1, ctx_max: int = 64, gemv2: bool = False,
                 threads: int | None = None):
        self._h = ctypes.c_void_p()
        t = threads or max(1, default_threads() // nranks)
        rc = ref_lib().ref_open(gguf_path.encode(), nranks, ctx_max, int(gemv2), t, ctypes.byref(self._h))
        if rc:
            raise RuntimeError(f"the reference runtime refused the model (rc {rc})")
        self.nranks = nranks

    def forward(self, token: int, pos: int) -> tuple[int, float]:
        t, v = ctypes.c_int(0), ctypes.c_float(0.0)
        rc = ref_lib().ref_forward(self._h, token, pos, ctypes.byref(t), ctypes.byref(v))
        if rc:
            raise RuntimeError(f"ref_forward failed ({rc})")
        return int(t.value), float(v.value)

    def read(self, what: int, n: int, rank: int = 0) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        if ref_lib().ref_read(self._h, what, rank, _ptr(out), n):
            raise RuntimeError("ref_read refused the size")
        return out

    def close(self) -> None:
        if self._h:
            ref_lib().ref_close(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
