"""llm-kv260 on B200: the Q4_0 x Q8_0 GEMV and the rank-ordered fp32
all-reduce of al-nafisah/llm-kv260's decode hot path, as sm_100a kernels
behind a C ABI (include/*.h) shaped like the reference's board/kv260gemv,
and the greedy decoder built on them (Decoder, include/b200_decoder.h).

The directory name has a hyphen, so it is loaded by path as module
``llm_kv260_b200`` (``__graft_entry__.load_package()``).
"""

from __future__ import annotations

from . import capi, gguf, model
from .capi import B200Error, lib
from .decoder import Decoder
from .gguf import GGUFFile
from .engine import LAYOUT_ROWS, LAYOUT_TILES, Engine, Gemv2Dev, GemvDev, QMat, Udmabuf, dev_ptr, tiled_bytes

__all__ = ["B200Error", "Decoder", "Engine", "GGUFFile", "Gemv2Dev", "GemvDev", "LAYOUT_ROWS", "LAYOUT_TILES", "QMat",
           "Udmabuf", "capi", "dev_ptr", "gguf", "lib", "model", "tiled_bytes"]
