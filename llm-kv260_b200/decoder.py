"""Python face of the greedy decoder (include/b200_decoder.h): the reference
runtime's decode loop (board/tp/tp_llama.cpp:783-968) on B200."""

from __future__ import annotations

import ctypes

import numpy as np

from . import capi
from .capi import check, lib


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


class Decoder:
    """One rank's decoder. `model` is a dict as model.synth_model returns (or a
    GGUF loader would): hparams, "layers", "token_embd", "output_norm"."""

    def __init__(self, model: dict | None, device: int = 0, rank: int = 0, nranks: int = 1, comm=None,
                 ctx_max: int = 512, kv_f16: bool = True, round_mode: int = 0, exact_norm: bool = False,
                 persistent: bool = False, _cfg=None):
        c = _cfg if _cfg is not None else capi.b200_decoder_config_t()
        if model is not None:
            for n in ("n_layer", "n_embd", "n_ff", "n_head", "n_head_kv", "head_dim", "n_vocab"):
                setattr(c, n, int(model[n]))
            c.rope_base, c.rms_eps = float(model["rope_base"]), float(model["rms_eps"])
        c.ctx_max, c.kv_f16, c.round_mode, c.exact_norm = ctx_max, int(kv_f16), round_mode, int(exact_norm)
        c.persistent = int(persistent)
        self.cfg, self.rank, self.nranks, self.ctx_max = c, rank, nranks, ctx_max
        self.h = ctypes.c_void_p()
        check(lib().b200_decoder_create(ctypes.byref(self.h), ctypes.byref(c), device, rank, nranks,
                                        comm.h if comm is not None else None), "b200_decoder_create")
        if model is None:
            return
        for i, L in enumerate(model["layers"]):
            arrs = [np.ascontiguousarray(L[n]) for n in ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate",
                                                        "ffn_up", "ffn_down")]
            norms = [np.ascontiguousarray(L[n], dtype=np.float32) for n in ("attn_norm", "ffn_norm")]
            check(lib().b200_decoder_set_layer(self.h, i, *[_p(a) for a in arrs], *[_p(a) for a in norms]),
                  "b200_decoder_set_layer")
        te = np.ascontiguousarray(model["token_embd"])
        on = np.ascontiguousarray(model["output_norm"], dtype=np.float32)
        check(lib().b200_decoder_set_output(self.h, _p(te), _p(on)), "b200_decoder_set_output")
        if model.get("rope_freqs") is not None:
            self.set_rope_freqs(model["rope_freqs"])

    @classmethod
    def from_gguf(cls, path: str, **kw) -> "Decoder":
        """A decoder for a GGUF Q4_0 model file (load_model, tp_llama.cpp:226-283):
        hyperparameters from its llama.* keys, every tensor loaded (and this
        rank's shard cut) through b200_decoder_load_gguf. Keyword arguments as
        for the constructor (device, rank, nranks, comm, ctx_max, ...)."""
        from .gguf import GGUFFile
        with GGUFFile(path) as g:
            dec = cls(None, _cfg=g.config(), **kw)
            try:
                check(lib().b200_decoder_load_gguf(dec.h, g.h), "b200_decoder_load_gguf")
            except Exception:
                dec.close()
                raise
        return dec

    def set_rope_freqs(self, freqs) -> None:
        """The model's rope_freqs factors (head_dim/2 floats), or None."""
        if freqs is None:
            check(lib().b200_decoder_set_rope_freqs(self.h, None), "b200_decoder_set_rope_freqs")
            return
        f = np.ascontiguousarray(freqs, dtype=np.float32)
        if f.shape != (self.cfg.head_dim // 2,):
            raise ValueError(f"rope_freqs must hold head_dim/2 = {self.cfg.head_dim // 2} factors")
        check(lib().b200_decoder_set_rope_freqs(self.h, _p(f)), "b200_decoder_set_rope_freqs")

    def forward(self, token: int, pos: int) -> tuple[int, float]:
        """runtime::forward + the greedy pick over all ranks."""
        t, v = ctypes.c_int32(0), ctypes.c_float(0.0)
        check(lib().b200_decoder_forward(self.h, token, pos, ctypes.byref(t), ctypes.byref(v)), "b200_decoder_forward")
        return int(t.value), float(v.value)

    def prefill(self, prompt) -> None:
        """Queue the prompt's forwards (no wait)."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        check(lib().b200_decoder_prefill(self.h, _p(p), p.shape[0]), "b200_decoder_prefill")

    def step(self, n: int = 1) -> None:
        """Queue n more forwards of the greedy loop (no wait)."""
        check(lib().b200_decoder_step(self.h, n), "b200_decoder_step")

    def generate(self, prompt, n_gen: int) -> tuple[np.ndarray, float, float]:
        """Greedy generate: (tokens, prompt_ms, gen_ms) -- device time of the
        prompt's forwards and of the remaining n_gen - 1."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(n_gen, dtype=np.int32)
        pm, gm = ctypes.c_double(0.0), ctypes.c_double(0.0)
        check(lib().b200_decoder_generate(self.h, _p(p), p.shape[0], n_gen, _p(out), ctypes.byref(pm),
                                          ctypes.byref(gm)), "b200_decoder_generate")
        return out, pm.value, gm.value

    def _read(self, what: int, n: int, dtype) -> np.ndarray:
        out = np.empty(n, dtype=dtype)
        check(lib().b200_decoder_read(self.h, what, _p(out), out.nbytes), "b200_decoder_read")
        return out

    def residual(self) -> np.ndarray:
        return self._read(0, self.cfg.n_embd, np.float32)

    def logits(self) -> np.ndarray:
        return self._read(1, self.cfg.n_vocab // self.nranks, np.float32)

    def tokens(self) -> np.ndarray:
        return self._read(2, self.ctx_max + 1, np.int32)

    def trace(self, tokens: int) -> None:
        """Persistent mode: stamp the phases of the first `tokens` tokens of each
        later launch. Graph mode (tokens 0 or 1): stamp every launch of the last
        token run."""
        check(lib().b200_decoder_trace(self.h, tokens), "b200_decoder_trace")
        self._trace_tokens = tokens

    def read_trace(self, nphases: int = 0, sms: int = 0) -> np.ndarray:
        """Persistent mode: [tokens, phases, SMs, 8] trace values (ns) of the last
        traced launch. Graph mode: [launches, 1024, 16] stamps of the last token
        (b200_decoder_trace)."""
        if not self.cfg.persistent:
            nl = 5 * self.cfg.n_layer + 1
            return self._read(7, nl * 1024 * 16, np.uint64).reshape(nl, 1024, 16)
        t = self._trace_tokens
        return self._read(7, t * nphases * sms * 8, np.uint64).reshape(t, nphases, sms, 8)

    def status(self) -> int:
        s = ctypes.c_uint(0)
        check(lib().b200_decoder_status(self.h, ctypes.byref(s)), "b200_decoder_status")
        return int(s.value)

    @property
    def stream(self) -> int:
        return int(lib().b200_decoder_stream(self.h) or 0)

    def close(self) -> None:
        if self.h:
            lib().b200_decoder_destroy(self.h)
            self.h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def rope_table(d: int, pos: int, base: float, freqs=None) -> np.ndarray:
    """The host RoPE table the decoder uploads (b200_rope_table[_freqs])."""
    cs = np.empty(d, dtype=np.float32)
    if freqs is None:
        check(lib().b200_rope_table(_p(cs), d, pos, base), "b200_rope_table")
    else:
        f = np.ascontiguousarray(freqs, dtype=np.float32)
        check(lib().b200_rope_table_freqs(_p(cs), d, pos, base, _p(f)), "b200_rope_table_freqs")
    return cs
