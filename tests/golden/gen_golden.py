"""Generate tests/golden/golden.json by running the REFERENCE contract itself.

    python tests/golden/gen_golden.py /path/to/reference

Imports ``llm_kv260.q4_0`` from the reference checkout named on the command
line and records
what it computes on the seeded inputs of ``cases.py``: the reference's own
golden digest, the gen_vectors.py cases, the Q8_0 rounding edges, and every
Llama-3.2-1B GEMV shape unsharded and K-split 2/4/8 ways with the rank-ordered
sum of board/tp/tp_llama.cpp:515-521. The reference does not travel to the GPU
box; the JSON does. Nothing here runs at test time.
"""

from __future__ import annotations

import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import cases  # noqa: E402


def load_reference(path: str):
    sys.path.insert(0, os.path.join(path, "src"))
    from llm_kv260 import q4_0  # noqa: E402
    return q4_0


def hexbytes(a: np.ndarray) -> str:
    return np.ascontiguousarray(a).tobytes().hex()


def main(ref_root: str) -> None:
    q = load_reference(ref_root)
    out: dict = {"contract_version": q.CONTRACT_VERSION, "generator": "tests/golden/gen_golden.py"}
    t0 = time.time()

    # The reference's golden vector (tests/test_q4_0_contract.py:184-191).
    w = cases.std_weights(96, 2048, 2024)
    x = cases.std_weights(1, 2048, 2025)[0]
    y = q.gemv_q4_0_f32(q.quantize_q4_0(w), 2048, x)
    assert cases.sha256(y) == cases.CONTRACT_GOLDEN_SHA256
    out["contract_golden"] = {"sha256_y": cases.sha256(y)}

    # gen_vectors.py cases.
    gv = []
    for k, rows, w, x in cases.gen_vector_inputs():
        blocks = q.quantize_q4_0(w)
        xq, xd = q.quantize_q8_0(x)
        y = q.gemv_q4_0(blocks, k, xq, xd)
        gv.append({"k": k, "rows": rows, "sha256_blocks": cases.sha256(blocks),
                   "sha256_xpacked": cases.sha256(q.pack_x_for_engine(xq, xd)), "y": hexbytes(y)})
    out["gen_vectors"] = gv

    # Q8_0 rounding edges and a random 8192-vector (test_q4_0_contract.py:42-59).
    edges = {}
    for name, xb in cases.q8_edge_inputs().items():
        xq, xd = q.quantize_q8_0(xb)
        edges[name] = {"q": xq.tolist(), "d_bits": xd.view(np.uint16).tolist()}
    out["q8_edges"] = edges
    xr = cases.std_weights(1, 8192, 1)[0]
    xq, xd = q.quantize_q8_0(xr)
    out["q8_random"] = {"sha256_q": cases.sha256(xq), "sha256_d": cases.sha256(xd)}

    # Codec (test_q4_0_contract.py:35-39, 62-66, 81-86).
    out["q4_codec"] = {
        "sha256_blocks_16x256_seed0": cases.sha256(q.quantize_q4_0(cases.std_weights(16, 256, 0))),
        "sha256_dequant_8x512_seed2": cases.sha256(q.dequantize_q4_0(q.quantize_q4_0(cases.std_weights(8, 512, 2)), 512)),
    }
    ints, d = q.unpack_q4_0(q.quantize_q4_0(cases.std_weights(8, 512, 2)), 512)
    out["q4_codec"]["sha256_unpack_ints_8x512_seed2"] = cases.sha256(ints)
    out["q4_codec"]["sha256_unpack_d_8x512_seed2"] = cases.sha256(d)

    # One lane per block (test_q4_0_contract.py:118-132) and the observable lane order (135-158).
    blocks = q.quantize_q4_0(cases.std_weights(4, 256, 7))
    xq, xd = q.quantize_q8_0(cases.std_weights(1, 256, 8)[0])
    out["one_lane"] = {"y": hexbytes(q.gemv_q4_0(blocks, 256, xq, xd))}
    blocks = q.quantize_q4_0(cases.std_weights(256, 2048, 9))
    xq, xd = q.quantize_q8_0(cases.std_weights(1, 2048, 10)[0])
    out["lane_order"] = {"sha256_y": cases.sha256(q.gemv_q4_0(blocks, 2048, xq, xd))}

    # BASELINE config 0 (full y) and config 1 (digests), with the K-split sums.
    name, n, k, seed = cases.CONFIG0
    blocks = q.quantize_q4_0(cases.shape_weights(n, k, seed))
    y = q.gemv_q4_0_f32(blocks, k, cases.shape_x(k, seed))
    out["config0"] = {"n": n, "k": k, "seed": seed, "sha256_blocks": cases.sha256(blocks), "y": hexbytes(y)}

    shapes = {}
    for name, n, k, seed in cases.LLAMA_1B_SHAPES:
        w = cases.shape_weights(n, k, seed)
        x = cases.shape_x(k, seed)
        blocks = q.quantize_q4_0(w)
        del w
        xq, xd = q.quantize_q8_0(x)
        y = q.gemv_q4_0(blocks, k, xq, xd)
        rec = {"n": n, "k": k, "seed": seed, "sha256_blocks": cases.sha256(blocks),
               "sha256_xpacked": cases.sha256(q.pack_x_for_engine(xq, xd)), "sha256_y": cases.sha256(y)}
        if name in cases.K_SPLIT:
            for parts in cases.SPLITS:
                kk = k // parts
                partials = []
                for r in range(parts):
                    sb = cases.k_slice_blocks(blocks, k, r, parts)
                    partials.append(q.gemv_q4_0_f32(sb, kk, x[r * kk:(r + 1) * kk]))
                s = partials[0].copy()
                for p in partials[1:]:
                    s = s + p
                rec[f"sha256_ksplit{parts}"] = cases.sha256(s)
        shapes[name] = rec
        print(f"{name}: {n}x{k} done ({time.time() - t0:.1f} s)", flush=True)
    out["shapes"] = shapes

    path = os.path.join(HERE, "golden.json")
    with open(path, "w") as fh:
        json.dump(out, fh, indent=1, sort_keys=True)
    print(f"wrote {path} in {time.time() - t0:.1f} s")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/gen_golden.py <path of the llm-kv260 reference checkout>")
    main(sys.argv[1])
