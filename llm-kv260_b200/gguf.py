"""Python face of include/b200_gguf.h: a GGUF Q4_0 model file as the
reference runtime's gguf_file reads it (board/tp/tp_llama.cpp:149-188)."""

from __future__ import annotations

import ctypes

import numpy as np

from . import capi
from .capi import check, lib

GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0 = 0, 1, 2, 8


class GGUFFile:
    """A mapped GGUF file (b200_gguf_open). Use as a context manager."""

    def __init__(self, path: str):
        self.h = ctypes.c_void_p()
        check(lib().b200_gguf_open(ctypes.byref(self.h), path.encode()), "b200_gguf_open")

    def config(self) -> capi.b200_decoder_config_t:
        """load_model's hyperparameters (tp_llama.cpp:228-236) as a decoder config."""
        c = capi.b200_decoder_config_t()
        check(lib().b200_gguf_config(self.h, ctypes.byref(c)), "b200_gguf_config")
        return c

    def hparams(self) -> dict:
        c = self.config()
        return {n: getattr(c, n) for n in ("n_layer", "n_embd", "n_ff", "n_head", "n_head_kv", "head_dim", "n_vocab",
                                           "rope_base", "rms_eps")}

    def tensor(self, name: str) -> tuple[np.ndarray, int, tuple[int, ...]]:
        """(bytes as a read-only uint8 view into the mapping, ggml type, ne)."""
        data, nbytes, typ = ctypes.c_void_p(), ctypes.c_uint64(0), ctypes.c_int(0)
        ne = (ctypes.c_int64 * 4)()
        check(lib().b200_gguf_tensor(self.h, name.encode(), ctypes.byref(data), ctypes.byref(nbytes),
                                     ctypes.byref(typ), ne), "b200_gguf_tensor")
        buf = (ctypes.c_uint8 * nbytes.value).from_address(data.value) if nbytes.value else None
        arr = np.frombuffer(buf, dtype=np.uint8) if buf is not None else np.empty(0, np.uint8)
        arr.flags.writeable = False
        return arr, typ.value, tuple(ne)

    def close(self) -> None:
        if self.h:
            lib().b200_gguf_close(self.h)
            self.h = ctypes.c_void_p()

    def __enter__(self) -> "GGUFFile":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
