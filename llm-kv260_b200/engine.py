"""Python wrappers over the C ABI: the engine (b200_engine.h) and the
drop-in device interfaces (gemv_dev.h, gemv2_dev.h, udmabuf.h).

Device memory comes from torch (plumbing only); every computation is a call
into libb200gemv.so.
"""

from __future__ import annotations

import ctypes

from . import capi
from .capi import check, lib

QK = 32
BLOCK_BYTES = 18
LAYOUT_ROWS = 0    # GGUF rows (B200_LAYOUT_ROWS)
LAYOUT_TILES = 1   # the engine's re-laid tiles (B200_LAYOUT_TILES)


def _torch():
    import torch
    return torch


def dev_ptr(t) -> int:
    """Device address of a CUDA tensor (or an int address as is)."""
    if isinstance(t, int):
        return t
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError("expected a contiguous tensor")
    return int(t.data_ptr())


def current_stream_handle(device: int) -> int:
    torch = _torch()
    return int(torch.cuda.current_stream(device).cuda_stream)


def tiled_bytes(rows: int, k: int) -> int:
    return int(lib().b200_tiled_bytes(rows, k))


class QMat:
    """A Q4_0 matrix in device memory (b200_qmat_t): GGUF rows, or the
    engine's tiles (Engine.repack)."""

    def __init__(self, blocks, rows: int, k: int, layout: int = LAYOUT_ROWS):
        if k % QK:
            raise ValueError(f"in_features must be a multiple of {QK}, got {k}")
        nbytes = rows * (k // QK) * BLOCK_BYTES if layout == LAYOUT_ROWS else tiled_bytes(rows, k)
        if hasattr(blocks, "numel") and blocks.numel() * blocks.element_size() < nbytes:
            raise ValueError(f"blocks tensor is smaller than the {nbytes} bytes of a {rows}x{k} matrix")
        self.blocks = blocks          # keeps the allocation alive
        self.rows, self.k, self.layout = rows, k, layout
        self.c = capi.b200_qmat_t(dev_ptr(blocks), rows, k, layout)

    @classmethod
    def from_numpy(cls, blocks_np, device: int = 0) -> "QMat":
        torch = _torch()
        rows, rb = blocks_np.shape
        t = torch.from_numpy(blocks_np.reshape(-1).copy()).to(f"cuda:{device}")
        return cls(t, rows, rb // BLOCK_BYTES * QK)

    @property
    def nbytes(self) -> int:
        """Algorithmic weight bytes (18 per 32 weights), whatever the layout."""
        return self.rows * (self.k // QK) * BLOCK_BYTES


class Engine:
    """b200_engine.h: the engine_t-level call (tp_llama.cpp:289-375)."""

    def __init__(self, device: int = 0, stream: int | None = None):
        self.device = device
        h = ctypes.c_void_p()
        check(lib().b200_engine_open(ctypes.byref(h), device), "b200_engine_open")
        self.h = h
        self.set_stream(current_stream_handle(device) if stream is None else stream)

    def close(self) -> None:
        if self.h:
            lib().b200_engine_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_stream(self, stream: int | None) -> None:
        check(lib().b200_engine_set_stream(self.h, stream), "b200_engine_set_stream")

    @property
    def stream(self) -> int:
        return int(lib().b200_engine_stream(self.h) or 0)

    def config(self) -> dict:
        c = capi.b200_engine_config_t()
        check(lib().b200_engine_get_config(self.h, ctypes.byref(c)), "b200_engine_get_config")
        return {f: getattr(c, f) for f, _ in c._fields_}

    def configure(self, **kw) -> None:
        c = capi.b200_engine_config_t()
        check(lib().b200_engine_get_config(self.h, ctypes.byref(c)), "b200_engine_get_config")
        for k, v in kw.items():
            if not hasattr(c, k):
                raise KeyError(k)
            setattr(c, k, int(v))
        check(lib().b200_engine_set_config(self.h, ctypes.byref(c)), "b200_engine_set_config")

    def gemv_f32(self, W: QMat, x, y, next: QMat | None = None) -> None:
        check(lib().b200_gemv_f32(self.h, ctypes.byref(W.c), dev_ptr(x), dev_ptr(y),
                                  ctypes.byref(next.c) if next else None), "b200_gemv_f32")

    def gemv_q8(self, W: QMat, xpacked, y, next: QMat | None = None) -> None:
        check(lib().b200_gemv_q8(self.h, ctypes.byref(W.c), dev_ptr(xpacked), dev_ptr(y),
                                 ctypes.byref(next.c) if next else None), "b200_gemv_q8")

    def quantize(self, x, xpacked, k: int) -> None:
        check(lib().b200_quantize_q8_0(self.h, dev_ptr(x), dev_ptr(xpacked), k), "b200_quantize_q8_0")

    def repack(self, W: QMat) -> QMat:
        """GGUF rows -> a new tiled matrix on this engine's device (b200_repack_q4_0)."""
        torch = _torch()
        if W.layout != LAYOUT_ROWS:
            raise ValueError("repack takes a GGUF-row matrix")
        n = tiled_bytes(W.rows, W.k)
        if n == 0:
            raise ValueError(f"cannot tile a {W.rows}x{W.k} matrix")
        dst = torch.empty(n, dtype=torch.uint8, device=f"cuda:{self.device}")
        check(lib().b200_repack_q4_0(self.h, W.c.w, W.rows, W.k, dev_ptr(dst)), "b200_repack_q4_0")
        return QMat(dst, W.rows, W.k, LAYOUT_TILES)

    def gemv_argmax_f32(self, W: QMat, x, y, out, index_base: int = 0) -> None:
        """gemv_f32 with the greedy pick over y fused into it (out: int32 index + index_base, float32 value)."""
        check(lib().b200_gemv_argmax_f32(self.h, ctypes.byref(W.c), dev_ptr(x), dev_ptr(y), index_base, dev_ptr(out)),
              "b200_gemv_argmax_f32")

    def argmax(self, y, n: int, out, index_base: int = 0) -> None:
        """First index of the largest of y[:n] (+ index_base) and its value -> out (8 bytes: int32, float32)."""
        check(lib().b200_argmax_f32(self.h, dev_ptr(y), n, index_base, dev_ptr(out)), "b200_argmax_f32")

    def capture_begin(self) -> None:
        check(lib().b200_capture_begin(self.h), "b200_capture_begin")

    def capture_end(self) -> "Graph":
        g = ctypes.c_void_p()
        check(lib().b200_capture_end(self.h, ctypes.byref(g)), "b200_capture_end")
        return Graph(self, g)

    def copy_async(self, dst: int, src: int, nbytes: int) -> None:
        check(lib().b200_copy_async(self.h, dst, src, nbytes), "b200_copy_async")

    def prefetch(self, W: QMat) -> None:
        check(lib().b200_prefetch(self.h, ctypes.byref(W.c)), "b200_prefetch")

    def sync(self, timeout_ms: int = 10000) -> None:
        check(lib().b200_engine_sync(self.h, timeout_ms), "b200_engine_sync")

    def status(self) -> int:
        s = ctypes.c_uint(0)
        check(lib().b200_engine_status(self.h, ctypes.byref(s)), "b200_engine_status")
        return int(s.value)

    def plan(self, rows: int, k: int, fused_f32: bool = False, layout: int = LAYOUT_TILES) -> tuple[int, int]:
        g, sm = ctypes.c_int(0), ctypes.c_int(0)
        check(lib().b200_gemv_plan(self.h, rows, k, layout, int(fused_f32), ctypes.byref(g), ctypes.byref(sm)),
              "b200_gemv_plan")
        return g.value, sm.value


class Graph:
    """A captured sequence of engine calls (b200_graph_t)."""

    def __init__(self, engine: Engine, handle):
        self.engine, self.h = engine, handle

    def launch(self) -> None:
        check(lib().b200_graph_launch(self.engine.h, self.h), "b200_graph_launch")

    def close(self) -> None:
        if self.h:
            lib().b200_graph_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class GemvDev:
    """gemv_dev.h: the reference's gemv_q4_0 engine interface (board/kv260gemv/gemv_dev.h)."""

    def __init__(self, name: str = "gemv_q4_0", quiet: bool = False):
        self.d = capi.gemv_dev_t()
        if lib().gemv_dev_open_named(ctypes.byref(self.d), name.encode(), int(quiet)) != 0:
            raise capi.B200Error(f"gemv_dev_open_named({name})", -1)

    def set_stream(self, stream: int | None) -> None:
        check(lib().gemv_dev_set_stream(ctypes.byref(self.d), stream), "gemv_dev_set_stream")

    def run(self, w: int, x: int, y: int, k: int, rows: int) -> None:
        check(lib().gemv_dev_run(ctypes.byref(self.d), w, x, y, k, rows), "gemv_dev_run")

    def start(self, w: int, x: int, y: int, k: int, rows: int) -> None:
        check(lib().gemv_dev_start(ctypes.byref(self.d), w, x, y, k, rows), "gemv_dev_start")

    def start4(self, w4, x: int, y: int, k: int, rows: int) -> None:
        arr = (ctypes.c_uint64 * 4)(*w4)
        check(lib().gemv_dev_start4(ctypes.byref(self.d), arr, x, y, k, rows), "gemv_dev_start4")

    def wait(self) -> None:
        check(lib().gemv_dev_wait(ctypes.byref(self.d)), "gemv_dev_wait")

    def close(self) -> None:
        lib().gemv_dev_close(ctypes.byref(self.d))


class Gemv2Dev:
    """gemv2_dev.h: fetch (L2 prefetch) + mac (GEMV) over the chunk-pair layout."""

    def __init__(self):
        self.d = capi.gemv2_dev_t()
        if lib().gemv2_dev_open(ctypes.byref(self.d)) != 0:
            raise capi.B200Error("gemv2_dev_open", -1)

    def fetch_start(self, w4, k: int, rows: int) -> None:
        arr = (ctypes.c_uint64 * 4)(*w4)
        check(lib().gemv2_fetch_start(ctypes.byref(self.d), arr, k, rows), "gemv2_fetch_start")

    def mac_start(self, x: int, y: int, k: int, rows: int) -> None:
        check(lib().gemv2_mac_start(ctypes.byref(self.d), x, y, k, rows), "gemv2_mac_start")

    def mac_wait(self) -> None:
        check(lib().gemv2_mac_wait(ctypes.byref(self.d)), "gemv2_mac_wait")

    def mac_idle(self) -> bool:
        return check(lib().gemv2_mac_idle(ctypes.byref(self.d)), "gemv2_mac_idle") == 1

    def drain(self) -> None:
        check(lib().gemv2_drain(ctypes.byref(self.d)), "gemv2_drain")

    def close(self) -> None:
        lib().gemv2_dev_close(ctypes.byref(self.d))


class Udmabuf:
    """udmabuf.h: device pool with a pinned host mirror (clean = H2D, invalidate = D2H)."""

    def __init__(self, name: str = "udmabuf0", size: int | None = None, device: int = 0):
        self.b = capi.udmabuf_t()
        if size is None:
            rc = lib().udmabuf_open(ctypes.byref(self.b), name.encode())
        else:
            rc = lib().udmabuf_open_size(ctypes.byref(self.b), name.encode(), size, device)
        if rc != 0:
            raise capi.B200Error(f"udmabuf_open({name})", rc)

    def alloc(self, size: int, align: int = 4096) -> int:
        """Host-mirror address of a new allocation (0 when the pool is full)."""
        return int(lib().udmabuf_alloc(ctypes.byref(self.b), size, align) or 0)

    def phys(self, host_addr: int) -> int:
        base = ctypes.cast(self.b.base, ctypes.c_void_p).value
        return self.b.phys + (host_addr - base)

    def view(self, host_addr: int, nbytes: int):
        """numpy uint8 view of the host mirror."""
        import numpy as np
        return np.ctypeslib.as_array((ctypes.c_uint8 * nbytes).from_address(host_addr))

    @staticmethod
    def clean(host_addr: int, nbytes: int) -> None:
        check(lib().udmabuf_clean(host_addr, nbytes), "udmabuf_clean")

    @staticmethod
    def invalidate(host_addr: int, nbytes: int) -> None:
        check(lib().udmabuf_invalidate(host_addr, nbytes), "udmabuf_invalidate")

    def close(self) -> None:
        lib().udmabuf_close(ctypes.byref(self.b))
