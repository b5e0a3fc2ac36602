"""ctypes declarations of the C ABI in include/*.h (libb200gemv.so).

The library is required: if it is not built, `lib()` raises. There is no CPU
path behind this module.
"""

from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libb200gemv.so")

c_int, c_uint, c_u64, c_size, c_vp, c_char_p = (ctypes.c_int, ctypes.c_uint, ctypes.c_uint64, ctypes.c_size_t,
                                                 ctypes.c_void_p, ctypes.c_char_p)


class gemv_dev_t(ctypes.Structure):
    """include/gemv_dev.h"""
    _fields_ = [("fd", c_int), ("stream", c_vp), ("done", c_vp), ("pending", c_int), ("owns_stream", c_int),
                ("timeout_ms", c_int), ("started_ns", c_u64)]


class gemv2_dev_t(ctypes.Structure):
    """include/gemv2_dev.h"""
    _fields_ = [("fetch", gemv_dev_t), ("mac", gemv_dev_t), ("w", c_u64 * 4), ("k", c_int), ("rows", c_int),
                ("fetched", c_int)]


class udmabuf_t(ctypes.Structure):
    """include/udmabuf.h"""
    _fields_ = [("fd", c_int), ("base", ctypes.POINTER(ctypes.c_uint8)), ("phys", c_u64), ("size", c_size),
                ("used", c_size)]


class b200_qmat_t(ctypes.Structure):
    """include/b200_engine.h"""
    _fields_ = [("w", c_u64), ("rows", c_int), ("k", c_int), ("layout", c_int)]


class b200_engine_config_t(ctypes.Structure):
    """include/b200_engine.h"""
    _fields_ = [("stage_bytes", c_int), ("stages", c_int), ("ctas_per_sm", c_int), ("l2_policy", c_int),
                ("pdl", c_int), ("round_mode", c_int), ("fuse_quantize", c_int), ("prefetch_next", c_int),
                ("xreg_chunks", c_int), ("kslices", c_int)]


P = ctypes.POINTER
class b200_decoder_config_t(ctypes.Structure):
    """include/b200_decoder.h"""
    _fields_ = [(n, c_int) for n in ("n_layer", "n_embd", "n_ff", "n_head", "n_head_kv", "head_dim", "n_vocab")] + \
               [("rope_base", ctypes.c_float), ("rms_eps", ctypes.c_float)] + \
               [(n, c_int) for n in ("ctx_max", "kv_f16", "round_mode", "exact_norm", "persistent")]


SIGNATURES: dict[str, tuple] = {
    # gemv_dev.h
    "gemv_dev_open": (c_int, [P(gemv_dev_t)]),
    "gemv_dev_open_named": (c_int, [P(gemv_dev_t), c_char_p, c_int]),
    "gemv_dev_close": (c_int, [P(gemv_dev_t)]),
    "gemv_dev_run": (c_int, [P(gemv_dev_t), c_u64, c_u64, c_u64, c_int, c_int]),
    "gemv_dev_start": (c_int, [P(gemv_dev_t), c_u64, c_u64, c_u64, c_int, c_int]),
    "gemv_dev_wait": (c_int, [P(gemv_dev_t)]),
    "gemv_dev_start4": (c_int, [P(gemv_dev_t), P(c_u64), c_u64, c_u64, c_int, c_int]),
    "gemv_dev_set_stream": (c_int, [P(gemv_dev_t), c_vp]),
    "gemv_dev_status": (c_int, [P(gemv_dev_t), P(c_uint)]),
    "gemv_dev_last_error": (c_char_p, []),
    # gemv2_dev.h
    "gemv2_dev_open": (c_int, [P(gemv2_dev_t)]),
    "gemv2_dev_close": (c_int, [P(gemv2_dev_t)]),
    "gemv2_fetch_start": (c_int, [P(gemv2_dev_t), P(c_u64), c_int, c_int]),
    "gemv2_fetch_wait": (c_int, [P(gemv2_dev_t)]),
    "gemv2_mac_start": (c_int, [P(gemv2_dev_t), c_u64, c_u64, c_int, c_int]),
    "gemv2_mac_wait": (c_int, [P(gemv2_dev_t)]),
    "gemv2_mac_idle": (c_int, [P(gemv2_dev_t)]),
    "gemv2_drain": (c_int, [P(gemv2_dev_t)]),
    # udmabuf.h
    "udmabuf_open": (c_int, [P(udmabuf_t), c_char_p]),
    "udmabuf_open_size": (c_int, [P(udmabuf_t), c_char_p, c_size, c_int]),
    "udmabuf_close": (c_int, [P(udmabuf_t)]),
    "udmabuf_alloc": (c_vp, [P(udmabuf_t), c_size, c_size]),
    "udmabuf_clean": (c_int, [c_vp, c_size]),
    "udmabuf_invalidate": (c_int, [c_vp, c_size]),
    # b200_engine.h
    "b200_engine_open": (c_int, [P(c_vp), c_int]),
    "b200_engine_close": (c_int, [c_vp]),
    "b200_engine_get_config": (c_int, [c_vp, P(b200_engine_config_t)]),
    "b200_engine_set_config": (c_int, [c_vp, P(b200_engine_config_t)]),
    "b200_engine_set_stream": (c_int, [c_vp, c_vp]),
    "b200_engine_stream": (c_vp, [c_vp]),
    "b200_gemv_f32": (c_int, [c_vp, P(b200_qmat_t), c_u64, c_u64, P(b200_qmat_t)]),
    "b200_gemv_q8": (c_int, [c_vp, P(b200_qmat_t), c_u64, c_u64, P(b200_qmat_t)]),
    "b200_quantize_q8_0": (c_int, [c_vp, c_u64, c_u64, c_int]),
    "b200_prefetch": (c_int, [c_vp, P(b200_qmat_t)]),
    "b200_engine_sync": (c_int, [c_vp, c_int]),
    "b200_engine_status": (c_int, [c_vp, P(c_uint)]),
    "b200_gemv_plan": (c_int, [c_vp, c_int, c_int, c_int, c_int, P(c_int), P(c_int)]),
    "b200_tiled_bytes": (c_u64, [c_int, c_int]),
    "b200_argmax_f32": (c_int, [c_vp, c_u64, c_int, c_int, c_u64]),
    "b200_argmax_f32_noalloc": (c_int, [c_u64, c_int, c_int, c_u64, c_vp]),
    "b200_gemv_argmax_f32": (c_int, [c_vp, P(b200_qmat_t), c_u64, c_u64, c_int, c_u64]),
    "b200_capture_begin": (c_int, [c_vp]),
    "b200_capture_end": (c_int, [c_vp, P(c_vp)]),
    "b200_graph_launch": (c_int, [c_vp, c_vp]),
    "b200_graph_destroy": (c_int, [c_vp]),
    "b200_copy_async": (c_int, [c_vp, c_u64, c_u64, c_u64]),
    "b200_repack_q4_0": (c_int, [c_vp, c_u64, c_int, c_int, c_u64]),
    "b200_device_count": (c_int, []),
    # b200_comm.h
    "b200_comm_create": (c_int, [P(c_vp), c_int, c_int, c_int, c_int]),
    "b200_comm_handle_bytes": (c_int, []),
    "b200_comm_export": (c_int, [c_vp, c_vp]),
    "b200_comm_import": (c_int, [c_vp, c_vp]),
    "b200_allreduce_sum": (c_int, [c_vp, c_u64, c_int, c_vp]),
    "b200_allgather": (c_int, [c_vp, c_u64, c_u64, c_int, c_vp]),
    "b200_allgather_pick": (c_int, [c_vp, c_u64, c_u64, c_vp]),
    "b200_comm_status": (c_int, [c_vp, P(c_uint)]),
    "b200_comm_destroy": (c_int, [c_vp]),
    # b200_decoder.h
    "b200_decoder_create": (c_int, [P(c_vp), P(b200_decoder_config_t), c_int, c_int, c_int, c_vp]),
    "b200_decoder_set_layer": (c_int, [c_vp, c_int] + [c_vp] * 9),
    "b200_decoder_set_output": (c_int, [c_vp, c_vp, c_vp]),
    "b200_decoder_forward": (c_int, [c_vp, c_int, c_int, P(ctypes.c_int32), P(ctypes.c_float)]),
    "b200_decoder_prefill": (c_int, [c_vp, c_vp, c_int]),
    "b200_decoder_step": (c_int, [c_vp, c_int]),
    "b200_decoder_generate": (c_int, [c_vp, c_vp, c_int, c_int, c_vp, P(ctypes.c_double), P(ctypes.c_double)]),
    "b200_decoder_read": (c_int, [c_vp, c_int, c_vp, c_u64]),
    "b200_decoder_status": (c_int, [c_vp, P(c_uint)]),
    "b200_decoder_trace": (c_int, [c_vp, c_int]),
    "b200_launch_floor": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, c_int, P(ctypes.c_float)]),
    "b200_rope_table": (c_int, [c_vp, c_int, c_int, ctypes.c_float]),
    "b200_rope_table_freqs": (c_int, [c_vp, c_int, c_int, ctypes.c_float, c_vp]),
    "b200_decoder_set_rope_freqs": (c_int, [c_vp, c_vp]),
    # b200_gguf.h
    "b200_gguf_open": (c_int, [P(c_vp), c_char_p]),
    "b200_gguf_close": (None, [c_vp]),
    "b200_gguf_config": (c_int, [c_vp, P(b200_decoder_config_t)]),
    "b200_gguf_tensor": (c_int, [c_vp, c_char_p, P(c_vp), P(c_u64), P(c_int), P(ctypes.c_int64)]),
    "b200_decoder_load_gguf": (c_int, [c_vp, c_vp]),
    "b200_decoder_stream": (c_vp, [c_vp]),
    "b200_decoder_destroy": (c_int, [c_vp]),
    "b200_last_error": (c_char_p, []),
}

_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """Load libb200gemv.so (built by llm-kv260_b200/build.py). Raises if absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is not built: run __graft_entry__.build() "
                               "(there is no CPU fallback for the GEMV)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        _lib = L
    return _lib


class B200Error(RuntimeError):
    """A C-ABI call returned a negative errno value."""

    def __init__(self, what: str, code: int):
        msg = lib().b200_last_error() or b""
        super().__init__(f"{what} failed ({code}): {msg.decode(errors='replace')}")
        self.code = code


def check(rc: int, what: str) -> int:
    if rc < 0:
        raise B200Error(what, rc)
    return rc
