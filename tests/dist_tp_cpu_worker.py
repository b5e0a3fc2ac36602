"""Worker for tests/test_tp_cpu.py (gloo, CPU, one process per rank): the
board/tp shard layout computed rank by rank with the CPU oracle, exchanged
with torch.distributed, summed in rank order -- it must give the digests the
reference contract gave for the same split (tests/golden/golden.json)."""

from __future__ import annotations

import datetime
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))

import cases  # noqa: E402
from oracle import oracle  # noqa: E402


def main() -> None:
    out_dir, mode = sys.argv[1], sys.argv[2]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=5))
    res = {}
    if mode == "shards":
        with open(os.path.join(ROOT, "tests", "golden", "golden.json")) as fh:
            golden = json.load(fh)
        for name, n, k, seed in cases.LLAMA_1B_SHAPES:
            if name == "lm_head":
                continue
            blocks = oracle.quantize_q4_0(cases.shape_weights(n, k, seed), threads=2)
            x = cases.shape_x(k, seed)
            if name in cases.K_SPLIT:
                kk = k // world        # attn_output / ffn_down: columns [r*K/n, (r+1)*K/n) (tp_llama.cpp:263-271)
                part = oracle.gemv_q4_0_f32(cases.k_slice_blocks(blocks, k, rank, world), kk,
                                            np.ascontiguousarray(x[rank * kk:(rank + 1) * kk]), threads=2)
                parts = [torch.zeros(n) for _ in range(world)]
                dist.all_gather(parts, torch.from_numpy(part))
                y = oracle.allreduce_ordered([p.numpy() for p in parts])
                res[name] = cases.sha256(y) == golden["shapes"][name][f"sha256_ksplit{world}"]
            else:
                rows = n // world      # q/k/v/gate/up: rows [r*N/n, (r+1)*N/n) (tp_llama.cpp:258-268)
                mine = oracle.gemv_q4_0_f32(blocks[rank * rows:(rank + 1) * rows], k, x, threads=2)
                parts = [torch.zeros(rows) for _ in range(world)]
                dist.all_gather(parts, torch.from_numpy(mine))
                res[name] = cases.sha256(np.concatenate([p.numpy() for p in parts])) == golden["shapes"][name]["sha256_y"]
    elif mode == "dropout":
        # rank 1 leaves between steps; rank 0's next collective must end with an error, not hang
        t = torch.ones(4)
        dist.all_reduce(t)
        if rank == 1:
            res["left"] = True
        else:
            try:
                dist.all_reduce(t)
                res["error"] = None
            except Exception as exc:   # gloo reports the missing peer after the group timeout
                res["error"] = type(exc).__name__
    with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as fh:
        json.dump(res, fh)
    if mode != "dropout":
        dist.destroy_process_group()
    os._exit(0)


if __name__ == "__main__":
    main()
