#!/usr/bin/env python
"""A small, fixed GEMV workload to put under a profiler.

Builds `--mats` seeded Q4_0 matrices of rows x k on one GPU (re-laid into the
engine's tile layout), then runs `--launches` fused-quantise GEMVs over them
round robin on the engine's stream, each GEMV's float32 input the previous
one's output head, so the launches are ordered as in a decode token. With
`--mats` chosen so that mats x rows x k x 18/32 bytes exceed the 126 MB L2,
every launch streams its weights from HBM. `--pick` fuses the greedy pick
into every launch (the lm_head form).

    python llm-kv260_b200/profile_case.py --rows 16384 --k 2048 --mats 8 --launches 12

Prints the mean device time per launch after the first round (CUDA events)
and exits 0.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def synth_q4_0(rows: int, k: int, seed: int) -> np.ndarray:
    """Uniform nibbles, float16 scales 0.0043 * U(0.75, 1.25): weights of
    about N(0, 0.02) in the GGUF Q4_0 row layout."""
    rng = np.random.default_rng(seed)
    nb = k // 32
    raw = rng.integers(0, 256, size=(rows * nb, 18), dtype=np.uint8)
    d = (0.0043 * (0.75 + 0.5 * rng.random(rows * nb))).astype(np.float16)
    raw[:, 0:2] = d.view(np.uint8).reshape(-1, 2)
    return raw.reshape(-1)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--rows", type=int, default=16384)
    ap.add_argument("--k", type=int, default=2048)
    ap.add_argument("--mats", type=int, default=8)
    ap.add_argument("--launches", type=int, default=12)
    ap.add_argument("--pick", type=int, default=0)
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--stages", type=int, default=8, help="shared-memory ring stages per CTA")
    args = ap.parse_args()
    if args.rows * args.k * 18 // 32 * args.mats > 4 << 30:
        raise SystemExit("profile case larger than 4 GB; keep profiler captures small")

    import torch
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    torch.cuda.set_device(args.device)
    dev = f"cuda:{args.device}"
    eng = pkg.Engine(args.device, stream=0)
    stream = torch.cuda.Stream(args.device)
    eng.set_stream(stream.cuda_stream)
    eng.configure(fuse_quantize=1, pdl=1, stages=args.stages, ctas_per_sm=4, kslices=1)
    mats = []
    for i in range(args.mats):
        t = torch.from_numpy(synth_q4_0(args.rows, args.k, 9000 + i)).to(dev)
        mats.append(eng.repack(pkg.QMat(t, args.rows, args.k)))
        eng.sync()
        del t
    f32 = dict(dtype=torch.float32, device=dev)
    x = torch.from_numpy(np.random.default_rng(1).standard_normal(max(args.k, args.rows)).astype(np.float32)).to(dev)
    ys = [torch.empty(max(args.k, args.rows), **f32) for _ in range(2)]
    sel = torch.zeros(2, dtype=torch.int32, device=dev)
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    src = x
    first = min(args.mats, args.launches - 1)   # the first round pays one-time set-up; time the rest
    with torch.cuda.stream(stream):
        for i in range(args.launches):
            if i == first:
                a.record(stream)
            W = mats[i % args.mats]
            dst = ys[i % 2]
            if args.pick:
                eng.gemv_argmax_f32(W, src[:args.k], dst[:args.rows], sel)
            else:
                eng.gemv_f32(W, src[:args.k], dst[:args.rows])
            src = dst if args.rows >= args.k else x
        b.record(stream)
    b.synchronize()
    if eng.status():
        raise SystemExit(f"engine status {eng.status()}")
    n = args.launches - first
    us = a.elapsed_time(b) * 1e3 / n
    gbs = (args.rows * args.k // 32 * 18 + 4 * args.k + 4 * args.rows) / us / 1e3
    print(f"{n} timed launches of {args.rows}x{args.k}: {us:.2f} us each, {gbs:.0f} GB/s")
    eng.close()


if __name__ == "__main__":
    main()
