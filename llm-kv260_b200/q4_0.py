"""The reference contract's GEMV functions (src/llm_kv260/q4_0.py), computed on
a B200 through the C ABI, with the reference's names, argument meaning and
errors (TypeError for a dtype, ValueError for a shape).

Inputs and outputs are numpy arrays, as in the reference; each call copies
them to and from the device, so this module is for checking and for callers
that hold host data. The decode loop uses the engine directly on device
buffers (engine.py).
"""

from __future__ import annotations

import numpy as np

from .engine import Engine, GemvDev

QK = 32                                     # q4_0.py:59
Q4_0_BYTES = 18                             # q4_0.py:60
LANES = 8                                   # q4_0.py:62
CONTRACT_VERSION = "llm-kv260/w4a8-q4_0-v2"  # q4_0.py:64

_engines: dict[int, Engine] = {}
_devs: dict[int, GemvDev] = {}


def _torch():
    import torch
    return torch


def engine(device: int = 0) -> Engine:
    if device not in _engines:
        _engines[device] = Engine(device)
    return _engines[device]


def _dev(device: int) -> GemvDev:
    if device not in _devs:
        _devs[device] = GemvDev(f"gemv_q4_0:{device}")
    return _devs[device]


def _to_dev(a: np.ndarray, device: int):
    torch = _torch()
    return torch.from_numpy(np.ascontiguousarray(a).reshape(-1).view(np.uint8).copy()).to(f"cuda:{device}")


def _check_blocks(blocks: np.ndarray, k: int) -> int:
    if blocks.dtype != np.uint8:
        raise TypeError(f"expected uint8 block bytes, got {blocks.dtype}")
    nb = k // QK
    if k % QK or blocks.ndim != 2 or blocks.shape[1] != nb * Q4_0_BYTES:
        raise ValueError(f"{blocks.shape[1] if blocks.ndim == 2 else blocks.shape} bytes per row is not "
                         f"{nb} blocks of {Q4_0_BYTES}")
    if nb % LANES:
        raise ValueError(f"{nb} blocks is not a multiple of {LANES} lanes")
    return blocks.shape[0]


def quantize_q8_0(x: np.ndarray, device: int = 0, round_mode: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """q4_0.py:83-97 on the GPU. Returns (q int8 [K], d float16 [K/32])."""
    if x.dtype != np.float32:
        raise TypeError(f"activations must be float32, got {x.dtype}")
    if x.ndim != 1 or x.shape[0] % QK:
        raise ValueError(f"x must be 1-D with a multiple of {QK} elements, got {x.shape}")
    torch = _torch()
    k = x.shape[0]
    e = engine(device)
    e.configure(round_mode=round_mode)
    xd_t = _to_dev(x, device)
    out = torch.empty(k + 4 * (k // QK), dtype=torch.uint8, device=f"cuda:{device}")
    e.quantize(xd_t, out, k)
    e.sync()
    host = out.cpu().numpy()
    e.configure(round_mode=0)
    return host[:k].view(np.int8).copy(), host[k:].view(np.float32).astype(np.float16)


def pack_x_for_engine(xq: np.ndarray, xd: np.ndarray) -> np.ndarray:
    """q4_0.py:193-200: the engine's activation buffer, int8[K] then float32[K/32]."""
    return np.concatenate([xq.view(np.uint8), xd.astype(np.float32).view(np.uint8)])


def gemv_q4_0(blocks: np.ndarray, k: int, xq: np.ndarray, xd: np.ndarray, device: int = 0) -> np.ndarray:
    """q4_0.py:151-182 on the GPU, through gemv_dev_run (gemv_dev.h:23)."""
    if xq.dtype != np.int8 or xd.dtype != np.float16:
        raise TypeError(f"x must be (int8, float16), got ({xq.dtype}, {xd.dtype})")
    n = _check_blocks(blocks, k)
    if xq.shape != (k,) or xd.shape != (k // QK,):
        raise ValueError(f"x shapes {xq.shape}, {xd.shape} do not match K={k}")
    torch = _torch()
    w_t = _to_dev(blocks, device)
    x_t = _to_dev(pack_x_for_engine(xq, xd), device)
    y_t = torch.empty(n, dtype=torch.float32, device=f"cuda:{device}")
    torch.cuda.synchronize(device)
    d = _dev(device)
    d.run(int(w_t.data_ptr()), int(x_t.data_ptr()), int(y_t.data_ptr()), k, n)
    return y_t.cpu().numpy()


def gemv_q4_0_f32(blocks: np.ndarray, k: int, x: np.ndarray, device: int = 0) -> np.ndarray:
    """q4_0.py:185-188 on the GPU, through the engine's call (b200_repack_q4_0 then b200_gemv_f32)."""
    if x.dtype != np.float32:
        raise TypeError(f"activations must be float32, got {x.dtype}")
    n = _check_blocks(blocks, k)
    if x.shape != (k,):
        raise ValueError(f"x shape {x.shape} does not match K={k}")
    torch = _torch()
    from .engine import QMat
    e = engine(device)
    W = e.repack(QMat(_to_dev(blocks, device), n, k))   # the engine re-lays weights at load
    x_t = _to_dev(x, device)
    y_t = torch.empty(n, dtype=torch.float32, device=f"cuda:{device}")
    e.gemv_f32(W, x_t, y_t)
    e.sync()
    return y_t.cpu().numpy()
